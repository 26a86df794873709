// tcg_quant.cuh -- per-tensor absmax quantisation fp32 -> int8 / packed int4 on
// the device: the producers of the integer GEMM's inputs.
//
// Replaces the reference's host loops quantize_absmax (src/data_int8.cu:74-89)
// and quantize_absmax_int4 (src/data_int4.cu:104-127) with three launches:
// an absmax reduction, the elementwise quantisation, and a one-thread kernel
// that publishes the scale.  Every float operation uses an explicitly rounded
// intrinsic (no contraction into FMA), so the codes and the scale are
// bit-identical to the reference's IEEE single-precision host arithmetic:
//   scale = absmax / Q;  inv = scale > 0 ? 1 / scale : 0;
//   q = clamp(x * inv, -Q, Q);  code = (int)(q >= 0 ? q + 0.5 : q - 0.5)
// with Q = 127 (int8) or 7 (int4, two codes per byte, low nibble = even k).
// HBM-bound: one read pass for the absmax, one read + 1/4 (int8) or 1/8
// (int4) write pass for the codes, walking the input backwards so that it
// starts on what the absmax pass left in L2.
#pragma once

#include <cstdint>

namespace tcg {

// |x| max over n floats into *absmax_bits (float bits, must start at +0).
// Non-negative floats order like their bit patterns as signed ints.  Four
// 16-byte loads in flight per thread per step.
__global__ void absmax_kernel(const float* __restrict__ x, long long n, int* __restrict__ absmax_bits)
{
    float m = 0.f;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    const long long n4 = n / 4;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < n4; i += 4 * stride) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = x4[i + u * stride];
#pragma unroll
        for (int u = 0; u < 4; ++u)
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w))));
    }
    for (; i < n4; i += stride) {
        const float4 v = x4[i];
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    for (long long j = n4 * 4 + static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += stride)
        m = fmaxf(m, fabsf(x[j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __shared__ float wmax[32];
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        m = threadIdx.x < (blockDim.x >> 5) ? wmax[threadIdx.x] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (threadIdx.x == 0) atomicMax(absmax_bits, __float_as_int(m));
    }
}

__device__ __forceinline__ float quant_inv(float absmax, float qmax)
{
    const float scale = __fdiv_rn(absmax, qmax);
    return scale > 0.f ? __fdiv_rn(1.f, scale) : 0.f;
}

__device__ __forceinline__ int quant_code(float x, float inv, float qmax)
{
    float q = __fmul_rn(x, inv);
    if (q > qmax) q = qmax;
    if (q < -qmax) q = -qmax;
    return __float2int_rz(q >= 0.f ? __fadd_rn(q, 0.5f) : __fsub_rn(q, 0.5f));
}

// The quantise passes walk the input from its end: the absmax pass just
// left the end of the input in L2, so the first part of this read hits there.
__device__ __forceinline__ uint32_t quant_word8(float4 v, float inv)
{
    return (static_cast<uint32_t>(quant_code(v.x, inv, 127.f)) & 0xFFu) |
           ((static_cast<uint32_t>(quant_code(v.y, inv, 127.f)) & 0xFFu) << 8) |
           ((static_cast<uint32_t>(quant_code(v.z, inv, 127.f)) & 0xFFu) << 16) |
           ((static_cast<uint32_t>(quant_code(v.w, inv, 127.f)) & 0xFFu) << 24);
}

__global__ void quantize_s8_kernel(const float* __restrict__ x, int8_t* __restrict__ out, long long n,
                                   const int* __restrict__ absmax_bits)
{
    const float inv = quant_inv(__int_as_float(*absmax_bits), 127.f);
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    const long long n4 = n / 4;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    uint32_t* o4 = reinterpret_cast<uint32_t*>(out);
    long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (; i + stride < n4; i += 2 * stride) {
        const long long j0 = n4 - 1 - i, j1 = n4 - 1 - (i + stride);
        const float4 v0 = x4[j0];
        const float4 v1 = x4[j1];
        o4[j0] = quant_word8(v0, inv);
        o4[j1] = quant_word8(v1, inv);
    }
    for (; i < n4; i += stride) {
        const long long j = n4 - 1 - i;
        o4[j] = quant_word8(x4[j], inv);
    }
    for (long long j = n4 * 4 + static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += stride)
        out[j] = static_cast<int8_t>(quant_code(x[j], inv, 127.f));
}

__device__ __forceinline__ uint32_t quant_byte4(float2 v, float inv)
{
    const int lo = quant_code(v.x, inv, 7.f);
    const int hi = quant_code(v.y, inv, 7.f);
    return static_cast<uint32_t>((lo & 0x0F) | ((hi & 0x0F) << 4));
}

// rows x cols_k floats -> rows x cols_k/2 bytes; byte = lo | hi << 4 with lo
// the code of the even column.  Eight floats (four output bytes) per step.
__global__ void quantize_s4_kernel(const float* __restrict__ x, int8_t* __restrict__ out, long long n_pairs,
                                   const int* __restrict__ absmax_bits)
{
    const float inv = quant_inv(__int_as_float(*absmax_bits), 7.f);
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    const long long n_g = n_pairs / 4;  // groups of 4 pairs: two float4 in, one 32-bit word out
    const float4* x4 = reinterpret_cast<const float4*>(x);
    uint32_t* o4 = reinterpret_cast<uint32_t*>(out);
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_g; i += stride) {
        const long long j = n_g - 1 - i;
        const float4 a = x4[2 * j];
        const float4 b = x4[2 * j + 1];
        o4[j] = quant_byte4(make_float2(a.x, a.y), inv) | (quant_byte4(make_float2(a.z, a.w), inv) << 8) |
                (quant_byte4(make_float2(b.x, b.y), inv) << 16) | (quant_byte4(make_float2(b.z, b.w), inv) << 24);
    }
    const float2* x2 = reinterpret_cast<const float2*>(x);
    for (long long j = n_g * 4 + static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; j < n_pairs; j += stride)
        out[j] = static_cast<int8_t>(quant_byte4(x2[j], inv));
}

// *scale = absmax / qmax, written over the absmax slot once every quantise
// block has read it (stream order).
__global__ void publish_scale_kernel(float* scale_and_absmax, float qmax)
{
    scale_and_absmax[0] = __fdiv_rn(scale_and_absmax[0], qmax);
}

}  // namespace tcg
