// tcg_gemm_kernel.cuh -- the one tcgen05 GEMM mainloop behind every precision.
//
// Replaces all of the reference's per-variant Ada kernels (kernels/fp16_*.cu,
// kernels/int8_*.cu and, after widening to int8, kernels/int4_*.cu) with one
// Blackwell-native design:
//
//   * tile shapes from 128 x 64 (one CTA) to 512 x 256 (a CTA pair issuing
//     tcgen05.mma.cta_group::2), grouped rasterisation (bands of tile-rows);
//   * scheduling: one cluster per work item, running clusters taking over
//     not-yet-started ones in launch order with cluster launch control (or,
//     for a single wave, persistent units round-robin);
//   * warp specialisation, 192 threads (int4: eight converter warps more,
//     widening packed operands in the ring stages):
//       warp 0 lane 0  -- TMA producer: 128-byte-swizzled A and B tiles into a
//                         kStages-deep shared-memory ring (full/empty
//                         mbarriers); in the leader CTA also the scheduler;
//       warp 1         -- allocates tensor memory; lane 0 issues tcgen05.mma
//                         into TMEM accumulators and releases ring slots with
//                         tcgen05.commit;
//       warps 2..5     -- epilogue, one per TMEM lane quarter: tcgen05.ld
//                         TMEM -> registers -> TMA store of C;
//   * every mbarrier wait is bounded: on expiry the kernel records a failure
//     word, drains its own copies in flight, frees TMEM and returns.
//
// One ring stage holds 128 bytes of K (64 fp16 or 128 int8 values) for the
// CTA's rows of A and of B.
#pragma once

#include <cuda_fp16.h>
#include "tcg_ptx.cuh"

namespace tcg {

constexpr int kBM = 128;        // UMMA M (one CTA, cta_group::1)
constexpr int kBKBytes = 128;   // bytes of K per ring stage (one swizzle row)
constexpr int kThreads = 192;   // 6 warps

constexpr uint32_t kErrWaitTimeout = 1;  // failure code in the high word
constexpr int kMaxExtraDst = 7;          // peer destinations of one GEMM's C

// Failure word, one per device.  This header is compiled into exactly one
// translation unit (tcgemm.cu), which owns the definition.
__device__ unsigned long long g_tcg_error_word = 0ull;

struct GemmParams {
    void* C;
    long long batch_stride_c;  // elements
    int M, N, K, batches;
    int tiles_m, tiles_n, num_kb;
    int group_m;               // tile-rows per rasterisation band
    int k_alternate;           // work items of odd waves walk K backwards (exact kinds only)
    int l2_a, l2_b;            // L2 eviction priority of A / B loads (l2_policy), -1 = no hint
    int n_extra;               // further destinations of C (peer GPUs' buffers), <= kMaxExtraDst
    void* extra[7];            // each receives the same tile at the same offset as C
    uint32_t idesc;            // tcgen05 instruction descriptor (make_idesc)
    const float* scale_a;      // non-null (int kinds): C = float(acc) * (*scale_a * *scale_b)
    const float* scale_b;
    int vec_store;             // C rows 16-byte aligned (N % 4 == 0, C aligned)
    int tma_store;             // write C through the tensor map (vec_store; peers then get plain stores)
    int split_from;            // work items from here on are column halves of the last tiles
    uint32_t idesc_half;       // instruction descriptor of a half (N = kBN / 2)
    int dynamic;               // 1: one cluster per work item, taken over by cluster launch control
    int wave_units;            // units (CTAs or pairs) resident at once
    unsigned long long timeout_ns;
    // stream-K split (two-CTA 512 x 256 tiles): unit u of sk_units takes
    // k-blocks [u*W/U, (u+1)*W/U) of the W = tiles * num_kb laid end to end
    int sk;
    int sk_units;
    long long sk_work;
    unsigned int sk_epoch;     // this launch's tag on the hand-off flags
    int sk_slot;               // this launch's row of flags
};

// Stream-K hand-off flags: a unit that computed the first k-blocks of a tile
// ("head") stores its raw accumulators into the tile's place in C, then sets
// its flag (one per CTA rank and epilogue warp) to the launch's tag; the
// unit that finishes the tile ("tail") waits for that flag, loads the
// partial back into tensor memory, resets the flag and continues.  Slots
// separate launches that may run at the same time.
constexpr int kSkSlots = 64;
constexpr int kSkMaxUnits = 256;
__device__ unsigned int g_sk_flag[kSkSlots * kSkMaxUnits * 8];

// A work item: tile t (or -1: no more work), k-blocks [kb0, kb1) of it, and
// what the unit does with its accumulators.
constexpr int kItemFull = 0;  // a whole tile: zero-initialised accumulate, store C
constexpr int kItemHead = 1;  // first k-blocks: store raw accumulators, signal
constexpr int kItemTail = 2;  // last k-blocks: load the head's partial first, store C
struct WorkItem {
    int t, kb0, kb1, kind, unit;
};

// Item i of stream-K unit u (false past its last).  A unit's range starts
// inside tile t0 at k-block x0 and ends inside tile t1 at x1; it runs the
// head of t1 first, then its whole tiles, then the tail of t0 last, so a
// tail's partial was produced at the very start of the previous unit.
__device__ __forceinline__ bool sk_item(const GemmParams& p, int u, int i, WorkItem& w)
{
    const long long kb = p.num_kb;
    const long long s = static_cast<long long>(u) * p.sk_work / p.sk_units;
    const long long e = static_cast<long long>(u + 1) * p.sk_work / p.sk_units;
    const int t0 = static_cast<int>(s / kb), x0 = static_cast<int>(s % kb);
    const int t1 = static_cast<int>(e / kb), x1 = static_cast<int>(e % kb);
    const int first_full = x0 ? t0 + 1 : t0;
    const int n_full = t1 > first_full ? t1 - first_full : 0;
    w.unit = u;
    if (x1) {
        if (i == 0) {
            w.t = t1, w.kb0 = 0, w.kb1 = x1, w.kind = kItemHead;
            return true;
        }
        --i;
    }
    if (i < n_full) {
        w.t = first_full + i, w.kb0 = 0, w.kb1 = p.num_kb, w.kind = kItemFull;
        return true;
    }
    if (x0 && i == n_full) {
        w.t = t0, w.kb0 = x0, w.kb1 = p.num_kb, w.kind = kItemTail;
        return true;
    }
    return false;
}

__device__ __forceinline__ unsigned int* sk_flag(const GemmParams& p, int unit, int slot_in_unit)
{
    return &g_sk_flag[(p.sk_slot * kSkMaxUnits + unit) * 8 + slot_in_unit];
}

// Tile shapes: one CTA per 128 x BN tile (single), a 2-CTA cluster per
// 256 x BN tile (pair, cta_group::2), one CTA per 256 x BN tile with two
// 128-row accumulators and no accumulator double buffering (wide), or a
// 2-CTA cluster per 512 x BN tile, each CTA holding 256 rows as two 128-row
// blocks and two accumulators (pair-wide).  Per MAC, pair and wide tiles
// stream 3/4 of the operand bytes of a single tile from L2, pair-wide tiles
// 9/16 (with BN = 256: 64 and 48 bytes per clock per SM at the int8 MMA
// rate).
constexpr int kShapeSingle = 0;
constexpr int kShapePair = 1;
constexpr int kShapeWide = 2;
constexpr int kShapePairWide = 3;

template <int kKind, bool kAccF16, bool kBMn, int kBN, int kStages, int kShape>
struct GemmTraits {
    static constexpr bool kPair = kShape == kShapePair || kShape == kShapePairWide;  // cta_group::2
    static constexpr bool kWide = kShape == kShapeWide || kShape == kShapePairWide;  // two A blocks per CTA
    // packed int4: TMA brings 64 bytes of packed K per row into a staging
    // ring; converter warps widen them into the int8 ring the MMAs read
    static constexpr bool kI4 = kKind == kKindI4;
    static constexpr int kElem = kKind == kKindF16 ? 2 : 1;
    static constexpr int kBK = kBKBytes / kElem;      // K elements per stage
    static constexpr int kUmmaK = 32 / kElem;         // K per instruction (32 bytes)
    static constexpr int kKSteps = kBK / kUmmaK;      // instructions per stage
    static constexpr int kASub = kWide ? 2 : 1;       // 128-row blocks of A per CTA
    static constexpr int kTileM = kBM * kASub * (kPair ? 2 : 1);  // rows of C per tile
    static constexpr int kUmmaM = kPair ? 2 * kBM : kBM;  // M of one MMA: 256 only with cta_group::2
    static constexpr int kBRows = kPair ? kBN / 2 : kBN;  // B rows (N) held by each CTA
    static constexpr int kASubBytes = kBM * kBKBytes;
    static constexpr int kABytes = kASub * kASubBytes;
    static constexpr int kBBytes = kBRows * kBKBytes;
    static constexpr int kStageBytes = kABytes + kBBytes;       // per CTA
    static constexpr int kTxBytes = kPair ? 2 * kStageBytes : kStageBytes;  // per leader barrier
    static constexpr int kAccBufs = kWide ? 1 : 2;    // TMEM accumulator buffers
    static constexpr int kTmemCols = 2 * kBN;         // (single/pair: 2 buffers; wide: 2 halves)
    // MN-major B arrives as kBRows/kAtomN boxes of kAtomN (128 bytes) x kBK rows.
    static constexpr int kAtomN = kBKBytes / kElem;
    static constexpr int kBoxBytesMn = kBK * kBKBytes;
    static constexpr int kEpiArrivals = kPair ? 8 : 4;  // one per epilogue warp (of both CTAs)
    static constexpr int kConvWarps = kI4 ? 8 : 0;       // int4 converter warps per CTA
    static constexpr int kThreadCount = kThreads + 32 * kConvWarps;
    static constexpr int kRing = 4;                      // work-item ring entries
    // arrivals per ring entry: the MMA issuer, every epilogue (and converter)
    // warp of both CTAs, and a pair's second producer (see the kernel)
    static constexpr int kRingConsumers = (kPair ? 10 : 5) + (kPair ? 2 : 1) * kConvWarps;
    // arrivals that fill an int8 ring stage: the TMA transaction (one arrive
    // with expect_tx); int4: every converter warp of the CTA, and for a pair
    // the leader's producer announcing the second CTA's 16-byte signal copy
    static constexpr int kFullArrivals = kI4 ? kConvWarps + (kPair ? 1 : 0) : 1;
    static constexpr int kSignalBytes = 16;  // int4 pair: second CTA's "stage converted" copy
    static constexpr int kBarrierBytes = 512;
    // two 32 x 32 word staging tiles (4 KB each) per epilogue warp
    static constexpr int kEpiStageBytes = 4 * 2 * 32 * 32 * 4;
    // int4: the TMA lands a stage's packed rows (64 bytes each) in the upper
    // half of the same ring stage; one barrier per stage counts those bytes
    static constexpr int kPkOffset = kStageBytes / 2;
    static constexpr int kPkStages = kI4 ? kStages : 0;
    static constexpr int kConvRows = kASub * kBM + kBRows;  // rows of a stage (A blocks, then B)
    static constexpr int kSmemBytes = kStages * kStageBytes + kEpiStageBytes + 1024 + kBarrierBytes;
    static_assert(kBRows % kAtomN == 0 || !kBMn, "MN-major B needs whole 128-byte atoms");
    static_assert(kTmemCols >= 32 && kTmemCols <= 512, "TMEM allocation");
    static_assert(kSmemBytes <= 232448, "shared memory per CTA");
    static_assert(!kI4 || (!kBMn && kConvRows % 32 == 0), "int4 staging");
    static constexpr int kRingInts = 4;  // t, kb0, kb1, kind | unit << 8
    static_assert(8 * (2 * kStages + 6 + 2 * kRing + kPkStages) + 8 + 4 * kRingInts * kRing <= 384, "barrier area");
};

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int group_m, int& b, int& tm,
                                            int& tn)
{
    const int per_batch = tiles_m * tiles_n;
    b = t / per_batch;
    const int r = t - b * per_batch;
    const int band = group_m * tiles_n;
    const int g = r / band;
    const int first_m = g * group_m;
    const int gsz = min(tiles_m - first_m, group_m);
    const int rr = r - g * band;
    tm = first_m + rr % gsz;
    tn = rr / gsz;
}

// Work item -> tile.  Items below split_from are whole tiles; from there on
// each remaining tile is cut into two column halves, consecutive items, so
// the last, partial wave of tiles becomes about half as long.
__device__ __forceinline__ void work_coords(int w, int split_from, int tiles_m, int tiles_n, int group_m, int& b,
                                            int& tm, int& tn, int& half)
{
    int t = w;
    half = -1;
    if (w >= split_from) {
        const int r = w - split_from;
        t = split_from + (r >> 1);
        half = r & 1;
    }
    tile_coords(t, tiles_m, tiles_n, group_m, b, tm, tn);
}

__device__ __forceinline__ void record_failure(volatile uint32_t* abort_flag, uint32_t detail)
{
    *abort_flag = 1u;
    __threadfence_block();
    atomicCAS(&g_tcg_error_word, 0ull,
              (static_cast<unsigned long long>(kErrWaitTimeout) << 32) | detail);
}

// One try_wait; kClusterScope: acquire at cluster scope (data written into
// this CTA's shared memory by the other CTA of its cluster).
template <bool kClusterScope = false>
__device__ __forceinline__ bool try_wait_scoped(uint32_t bar, uint32_t parity)
{
    return kClusterScope ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity);
}

// Single-thread bounded wait.  true: the phase of `parity` completed.
// false: this CTA is aborting (this wait expired, or another role's did).
template <bool kClusterScope = false>
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag,
                                             unsigned long long timeout_ns, uint32_t detail)
{
    if (try_wait_scoped<kClusterScope>(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (try_wait_scoped<kClusterScope>(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_timer_ns() - t0 > timeout_ns) {
            record_failure(abort_flag, detail);
            return false;
        }
    }
}

// Whole-warp bounded wait with a warp-uniform result.  A completed phase is
// sticky until every waiter has arrived for the next one, so once any lane
// sees completion all lanes will.
template <bool kClusterScope = false>
__device__ __forceinline__ bool wait_bounded_warp(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag,
                                                  unsigned long long timeout_ns, uint32_t detail)
{
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
        const bool ok = try_wait_scoped<kClusterScope>(bar, parity);
        if (__all_sync(0xffffffffu, ok)) return true;
        if (__any_sync(0xffffffffu, ok)) continue;
        if (i == 0) t0 = global_timer_ns();
        const bool ab = (*abort_flag != 0u);
        const bool expired = (global_timer_ns() - t0) > timeout_ns;
        const unsigned stop = __ballot_sync(0xffffffffu, ab || expired);
        if (stop) {
            if ((threadIdx.x & 31) == (__ffs(stop) - 1) && !ab) record_failure(abort_flag, detail);
            return false;
        }
    }
}

// Bounded drain wait used only on the abort path (ignores the abort flag).
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity)
{
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_timer_ns() - t0 > 200000000ull) return;  // 200 ms
    }
}

__device__ __forceinline__ uint32_t cluster_id_x()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t num_clusters_x()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}

// Convert 32 accumulator words in place: fp16 accumulators (low halves) to
// fp32, or int32 to fp32 scaled by the combined dequantisation factor.
// kScaled16: int4 accumulators hold 256 x the product (both operands were
// widened as 16 x value, see spread_word); the exact result is acc >> 8.
template <bool kAccF16, bool kScaled16 = false>
__device__ __forceinline__ void epi_convert(uint32_t (&v)[32], bool dequant, float combined)
{
    if constexpr (kScaled16) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = static_cast<uint32_t>(static_cast<int32_t>(v[j]) >> 8);
    }
    if constexpr (kAccF16) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            v[j] = __float_as_uint(__half2float(__ushort_as_half(static_cast<unsigned short>(v[j] & 0xFFFFu))));
    }
    if (dequant) {  // (float)acc * (scale_a * scale_b), one rounding each
#pragma unroll
        for (int j = 0; j < 32; ++j)
            v[j] = __float_as_uint(__fmul_rn(__int2float_rn(static_cast<int>(v[j])), combined));
    }
}

// One 32 x 32 word block of C (lane i holds row i) out through a TMA store:
// into a staging tile in the tensor map's 128-byte swizzle (16-byte chunk q
// of row r at chunk q ^ (r & 7): no bank conflicts), then one bulk store.
// Two staging tiles per warp alternate; before one is rewritten, the store
// that last read it (two stores ago) must have finished reading.
__device__ __forceinline__ void epi_store_tma(const CUtensorMap* tmC, uint32_t* buf, uint32_t buf_s,
                                              const uint32_t (&v)[32], int lane, int col, int row, int b,
                                              bool reduce = false)
{
    if (lane == 0) bulk_wait_group_read<1>();
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 8; ++q)
        *reinterpret_cast<uint4*>(buf + lane * 32 + ((q ^ (lane & 7)) << 2)) =
            make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        if (reduce)
            tma_reduce_add_3d(tmC, buf_s, col, row, b);
        else
            tma_store_3d(tmC, buf_s, col, row, b);
        bulk_commit_group();
    }
}

// The same 32 x 32 block, read back from its staging tile, to every peer
// destination (the epilogue all-gather): plain 16-byte stores over NVLink,
// 4 rows x 128 bytes per instruction.  C rows are 16-byte aligned here.
__device__ __forceinline__ void epi_store_peers(const GemmParams& p, const uint32_t* buf, int row0, int col,
                                                long long cbase, int lane)
{
    const int rsub = lane >> 3;
    const int gcol = col + (lane & 7) * 4;
#pragma unroll 2
    for (int it = 0; it < 8; ++it) {
        const int r = it * 4 + rsub;
        const uint4 w = *reinterpret_cast<const uint4*>(buf + r * 32 + (((lane & 7) ^ (r & 7)) << 2));
        const int grow = row0 + r;
        if (grow < p.M && gcol < p.N) {
            const long long off = cbase + static_cast<long long>(grow) * p.N + gcol;
#pragma unroll 1
            for (int d = 0; d < p.n_extra; ++d)
                *reinterpret_cast<uint4*>(static_cast<uint32_t*>(p.extra[d]) + off) = w;
        }
    }
}

// Widen four packed int4 bytes (two values per byte, low nibble first) to
// eight int8 values.  A nibble x (two's complement, 4 bits) has the value
// (x ^ 8) - 8.  With x ^ 0x88 every byte lies in [0x80, 0x8f], so subtracting
// 0x08 from all four bytes at once borrows across none of them and leaves
// 0x80 + value; the final ^ 0x80 (after interleaving) removes the bias.  Nine
// integer operations for eight values (no byte-SIMD emulation).
__device__ __forceinline__ void widen_word(uint32_t w, uint32_t& o0, uint32_t& o1)
{
    const uint32_t lo = ((w & 0x0F0F0F0Fu) ^ 0x88888888u) - 0x08080808u;
    const uint32_t hi = (((w >> 4) & 0x0F0F0F0Fu) ^ 0x88888888u) - 0x08080808u;
    o0 = __byte_perm(lo, hi, 0x5140) ^ 0x80808080u;  // lo0 hi0 lo1 hi1
    o1 = __byte_perm(lo, hi, 0x7362) ^ 0x80808080u;  // lo2 hi2 lo3 hi3
}

// The converter's widening: four packed bytes (eight int4 values, k = 0..7,
// low nibble first) become two words of int8 holding 16 x value -- the even
// k (low nibbles shifted into the high half of each byte) in `ev`, the odd k
// (high nibbles, masked in place) in `od`.  Two's-complement nibbles need no
// sign extension this way (the nibble's sign bit is the byte's), three
// integer operations for eight values.  Both operands go through the same
// function, so the K order inside each 32-value group is the same permutation
// for A and B and the dot products are unchanged; every product is 256 x the
// int4 product, which the epilogue divides out exactly (acc >> 8).  The
// int32 accumulator holds K x 2^14 at most: K < 131072.
__device__ __forceinline__ void spread_word(uint32_t w, uint32_t& ev, uint32_t& od)
{
    ev = (w << 4) & 0xF0F0F0F0u;
    od = w & 0xF0F0F0F0u;
}

// int4 stage conversion, in place, by the kConv threads of the converter
// warps (thread ct).  The TMA put the stage's `rows` packed rows (64 bytes =
// 128 K values each, back to back) in the upper half of the ring stage; they
// are spread (spread_word) into the whole stage in the layout a
// 128-byte-swizzled TMA load
// would have produced (row r at r * 128, 16-byte chunk c stored at chunk
// c ^ (r & 7)), which the MMA descriptors read.  Phase 1 (conv_load) reads
// each thread's packed chunks into registers; after a barrier of the
// converter warps, phase 2 (conv_store) writes them, so no write reaches
// packed bytes another thread has yet to read.  Every 8 consecutive threads
// read two consecutive packed rows (128 contiguous bytes) and write chunks of
// two rows whose swizzled positions are disjoint: no bank conflicts.
template <int kConv, int kMaxRows>
struct ConvPlan {
    static constexpr int kStep = kConv >= 4 ? kConv / 4 : 1;  // rows per pass
    static constexpr int kPasses = (kMaxRows + kStep - 1) / kStep;
};

template <int kConv, int kMaxRows>
__device__ __forceinline__ void conv_load(const uint8_t* src, int rows, int ct,
                                          uint4 (&v)[ConvPlan<kConv, kMaxRows>::kPasses])
{
    using P = ConvPlan<kConv, kMaxRows>;
    const int j = ct & 3;
#pragma unroll
    for (int u = 0; u < P::kPasses; ++u) {
        const int r = u * P::kStep + (ct >> 2);
        if (r < rows) v[u] = *reinterpret_cast<const uint4*>(src + r * 64 + j * 16);
    }
}

template <int kConv, int kMaxRows>
__device__ __forceinline__ void conv_store(uint8_t* dst, int rows, int ct,
                                           const uint4 (&v)[ConvPlan<kConv, kMaxRows>::kPasses])
{
    using P = ConvPlan<kConv, kMaxRows>;
    const int j = ct & 3;  // 16-byte packed chunk = int8 chunks 2j, 2j+1
#pragma unroll
    for (int u = 0; u < P::kPasses; ++u) {
        const int r = u * P::kStep + (ct >> 2);
        if (r < rows) {
            uint4 a, b;
            spread_word(v[u].x, a.x, a.y);
            spread_word(v[u].y, a.z, a.w);
            spread_word(v[u].z, b.x, b.y);
            spread_word(v[u].w, b.z, b.w);
            uint8_t* row = dst + r * 128;
            const int sw = r & 7;
            *reinterpret_cast<uint4*>(row + (((2 * j) ^ sw) << 4)) = a;
            *reinterpret_cast<uint4*>(row + (((2 * j + 1) ^ sw) << 4)) = b;
        }
    }
}

// kPair = false: one CTA per 128 x kBN tile, tcgen05 cta_group::1.
// kPair = true : a cluster of two CTAs per 256 x kBN tile, tcgen05
//   cta_group::2.  CTA r holds rows [128r, 128r+128) of A and columns
//   [r*kBN/2, (r+1)*kBN/2) of B; the leader (rank 0) issues every MMA, which
//   reads both CTAs' shared memory and writes rows 128r.. of D into CTA r's
//   tensor memory.  Both CTAs' TMA loads complete on the leader's full
//   barriers; the leader's commits arrive on both CTAs' empty / tmem-full
//   barriers; both epilogues release the accumulator on the leader's barrier.
template <int kKind, bool kAccF16, bool kBMn, int kBN, int kStages, int kShape>
__global__ void __launch_bounds__(GemmTraits<kKind, kAccF16, kBMn, kBN, kStages, kShape>::kThreadCount, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmC,
                const GemmParams p)
{
    using T = GemmTraits<kKind, kAccF16, kBMn, kBN, kStages, kShape>;
    constexpr bool kPair = T::kPair;
    constexpr bool kWide = T::kWide;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint32_t* epi_stage = reinterpret_cast<uint32_t*>(smem + kStages * T::kStageBytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(epi_stage) + T::kEpiStageBytes);
    uint64_t* full = bars;
    uint64_t* empty = bars + kStages;
    uint64_t* tfull = bars + 2 * kStages;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint64_t* qfull = drain + 1;          // work-item ring: entry published
    uint64_t* qempty = qfull + T::kRing;  // work-item ring: entry read by every consumer (leader CTA's)
    uint64_t* clcbar = qempty + T::kRing; // cluster launch control response landed
    uint64_t* full_pk = clcbar + 1;       // int4: a stage's packed rows landed (TMA, this CTA)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(full_pk + T::kPkStages);
    volatile uint32_t* abort_flag = tmem_slot + 1;
    volatile int* ring = reinterpret_cast<volatile int*>(tmem_slot + 2);
    const uint32_t clc_resp = smem_u32(reinterpret_cast<uint8_t*>(bars) + 384);  // 16 bytes, 16-aligned
    const uint32_t sig_buf = smem_u32(reinterpret_cast<uint8_t*>(bars) + 400);   // 16 bytes, 16-aligned

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = kPair ? cluster_ctarank() : 0u;
    const bool leader = (rank == 0u);
    // this unit's first work item: its own index (one cluster per work item
    // with cluster launch control, one per resident unit otherwise)
    const int unit = kPair ? static_cast<int>(cluster_id_x()) : static_cast<int>(blockIdx.x);
    const int units = kPair ? static_cast<int>(num_clusters_x()) : static_cast<int>(gridDim.x);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&full[s]), T::kFullArrivals);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int s = 0; s < T::kPkStages; ++s) mbar_init(smem_u32(&full_pk[s]), 1);
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&tfull[a]), 1);
            mbar_init(smem_u32(&tempty[a]), T::kEpiArrivals);
        }
        mbar_init(smem_u32(drain), 1);
        for (int r = 0; r < T::kRing; ++r) {
            mbar_init(smem_u32(&qfull[r]), 1);
            mbar_init(smem_u32(&qempty[r]), T::kRingConsumers);
        }
        mbar_init(smem_u32(clcbar), 1);
        *abort_flag = 0u;
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        if constexpr (kPair) {
            tmem_alloc_pair(smem_u32(tmem_slot), T::kTmemCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(tmem_slot), T::kTmemCols);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (kPair) cluster_sync_all();  // the peer's barriers exist before any remote arrival
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Everything above overlaps the previous kernel's tail; global memory is
    // touched only below.
    grid_dependency_wait();
    grid_launch_dependents();

    const int num_tiles = p.tiles_m * p.tiles_n * p.batches;
    const int num_work = p.split_from + 2 * (num_tiles - p.split_from);
    const uint32_t stage0 = smem_u32(smem);
    // producer bookkeeping for the abort drain: per stage, a load was issued /
    // the parity of its phase; a cluster-launch-control response in flight
    uint32_t issued = 0, issued_parity = 0;
    bool signalled = false;  // int4 pair, second CTA: a signal copy into the leader was sent
    bool clc_pending = false;
    uint32_t clc_phase = 0;

    // Work items reach every role through a ring of kRing entries in shared
    // memory.  Thread 0 of the leader CTA (the scheduler) publishes each item
    // -- into both CTAs' rings for a pair -- and -1 after the last; the
    // consumers (the MMA issuer, every epilogue warp, and a pair's second
    // producer) each arrive on the leader's entry-empty barrier once they
    // have read it.
    int q = 0;
    uint32_t qph = 0;
    const auto ring_next = [&]() {
        if (++q == T::kRing) {
            q = 0;
            qph ^= 1u;
        }
    };
    // Entry q holds a WorkItem as four ints.  The scheduler writes it into
    // this CTA's ring and, for a pair, the peer's (then arrives on both
    // entry-full barriers; cluster-scope release for the peer's copy).
    const auto ring_put = [&](const WorkItem& w) {
        const int e[4] = {w.t, w.kb0, w.kb1, w.kind | (w.unit << 8)};
#pragma unroll
        for (int i = 0; i < T::kRingInts; ++i) ring[q * T::kRingInts + i] = e[i];
        if constexpr (kPair) {
#pragma unroll
            for (int i = 0; i < T::kRingInts; ++i)
                st_cluster_u32(mapa_shared(smem_u32((const void*)&ring[q * T::kRingInts + i]), 1),
                               static_cast<uint32_t>(e[i]));
            mbar_arrive_cluster_release(mapa_shared(smem_u32(&qfull[q]), 1));
        }
        mbar_arrive(smem_u32(&qfull[q]));
    };
    const auto ring_get = [&]() {
        WorkItem w;
        w.t = ring[q * T::kRingInts + 0];
        w.kb0 = ring[q * T::kRingInts + 1];
        w.kb1 = ring[q * T::kRingInts + 2];
        const int ku = ring[q * T::kRingInts + 3];
        w.kind = ku & 0xFF;
        w.unit = ku >> 8;
        return w;
    };
    // a consumer has read entry q: release it on the leader's barrier.  The
    // read it releases is of this CTA's own shared memory and its value is
    // already in a register, so a CTA-scope release suffices; a
    // cluster-scope one would stall the thread about a microsecond per item.
    const auto ring_release = [&]() {
        if constexpr (kPair) {
            if (leader)
                mbar_arrive(smem_u32(&qempty[q]));
            else
                mbar_arrive_cluster(mapa_shared(smem_u32(&qempty[q]), 0));
        } else {
            mbar_arrive(smem_u32(&qempty[q]));
        }
    };

    if (threadIdx.x == 0) {
        // ------------------------------------------------ TMA producer ----
        int stage = 0;
        uint32_t phase = 0;
        bool aborted = false;
        int local = 0;
        const bool hint = p.l2_a >= 0 || p.l2_b >= 0;
        const uint64_t pol_a = l2_policy(p.l2_a);
        const uint64_t pol_b = l2_policy(p.l2_b);
        bool clc_live = p.dynamic != 0;  // the grid may still hold clusters to take over
        int t = unit;
        int sk_i = 0;  // stream-K: this unit's next item
        WorkItem cur{t, 0, p.num_kb, kItemFull, unit};
        if (p.sk && !sk_item(p, unit, 0, cur)) cur.t = -1;
        for (;; ++local) {
            if (leader) {
                // publish the item (scheduler)
                if (!wait_bounded(smem_u32(&qempty[q]), qph ^ 1u, abort_flag, p.timeout_ns,
                                  (blockIdx.x << 8) | 0x70u | q)) {
                    aborted = true;
                    break;
                }
                ring_put(cur);
                ring_next();
                if (cur.t < 0) break;
                if (clc_live) {  // ask for the next work item now; the answer is read after this tile's loads
                    mbar_arrive_expect_tx(smem_u32(clcbar), 16);
                    clc_try_cancel(clc_resp, smem_u32(clcbar));
                    clc_pending = true;
                }
            } else {
                // a pair's second producer follows the leader's ring
                if (!wait_bounded<true>(smem_u32(&qfull[q]), qph, abort_flag, p.timeout_ns,
                                        (blockIdx.x << 8) | 0x78u | q)) {
                    aborted = true;
                    break;
                }
                cur = ring_get();
                ring_release();
                ring_next();
                if (cur.t < 0) break;
            }
            t = cur.t;
            int b, tm, tn, half;
            work_coords(t, p.split_from, p.tiles_m, p.tiles_n, p.group_m, b, tm, tn, half);
            const int a_row = tm * T::kTileM + static_cast<int>(rank) * (T::kASub * kBM);
            // a half tile: columns [half * kBN/2, +kBN/2) of the tile, each
            // CTA of a pair holding half of those
            const int b_row = half < 0 ? tn * kBN + static_cast<int>(rank) * T::kBRows
                                       : tn * kBN + half * (kBN / 2) + static_cast<int>(rank) * (T::kBRows / 2);
            const uint32_t tx = half < 0 ? T::kTxBytes : T::kTxBytes - (kPair ? 2 : 1) * (T::kBBytes / 2);
            const int b_atoms = half < 0 ? T::kBRows / T::kAtomN : T::kBRows / T::kAtomN / 2;
            const CUtensorMap* mapB = half < 0 ? &tmB : &tmBh;
            // The items in flight (about one wave: wave_units consecutive
            // items) finish at about the same K.  Walking K backwards on every
            // other wave starts each wave on the K range the previous wave just
            // brought into L2.  Integer accumulation is exact in any order;
            // floating-point kinds keep one order.
            const bool reverse = p.k_alternate && ((t / p.wave_units) & 1);
            for (int kb = cur.kb0; kb < cur.kb1; ++kb) {
                const int kc = reverse ? cur.kb0 + cur.kb1 - 1 - kb : kb;
                if constexpr (T::kI4) {
                    // packed rows (64 bytes of K each) into the upper half of
                    // this CTA's ring stage once the MMAs have released it,
                    // completing on this CTA's barrier: the converter warps of
                    // the same CTA widen them in place
                    if (!wait_bounded(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, p.timeout_ns,
                                      (blockIdx.x << 8) | 0x10u | stage)) {
                        aborted = true;
                        break;
                    }
                    if (kPair && leader)  // the second CTA's converters signal with a 16-byte copy
                        mbar_arrive_expect_tx(smem_u32(&full[stage]), T::kSignalBytes);
                    const uint32_t fb = smem_u32(&full_pk[stage]);
                    const uint32_t dst = stage0 + stage * T::kStageBytes + T::kPkOffset;
                    const int b_rows = half < 0 ? T::kBRows : T::kBRows / 2;
                    mbar_arrive_expect_tx(fb, static_cast<uint32_t>((T::kASub * kBM + b_rows) * 64));
#pragma unroll
                    for (int h = 0; h < T::kASub; ++h)
                        tma_load_3d(dst + h * kBM * 64, &tmA, fb, kc * 64, a_row + h * kBM, b);
                    tma_load_3d(dst + T::kASub * kBM * 64, mapB, fb, kc * 64, b_row, b);
                    issued |= 1u << stage;
                    issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                    continue;
                }
                const uint32_t fb_local = smem_u32(&full[stage]);
                if (!wait_bounded(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, p.timeout_ns,
                                  (blockIdx.x << 8) | 0x10u | stage)) {
                    aborted = true;
                    break;
                }
                const uint32_t a_dst = stage0 + stage * T::kStageBytes;
                const uint32_t b_dst = a_dst + T::kABytes;
                if constexpr (kPair) {
                    const uint32_t fb = mapa_shared(fb_local, 0);  // the leader's full barrier
                    if (leader) mbar_arrive_expect_tx(fb_local, tx);
#pragma unroll
                    for (int h = 0; h < T::kASub; ++h) {
                        if (hint)
                            tma_load_3d_pair_hint(a_dst + h * T::kASubBytes, &tmA, fb, kc * T::kBK, a_row + h * kBM,
                                                  b, pol_a);
                        else
                            tma_load_3d_pair(a_dst + h * T::kASubBytes, &tmA, fb, kc * T::kBK, a_row + h * kBM, b);
                    }
                    if constexpr (kBMn) {
#pragma unroll 1
                        for (int j = 0; j < b_atoms; ++j) {
                            if (hint)
                                tma_load_3d_pair_hint(b_dst + j * T::kBoxBytesMn, &tmB, fb,
                                                      b_row + j * T::kAtomN, kc * T::kBK, b, pol_b);
                            else
                                tma_load_3d_pair(b_dst + j * T::kBoxBytesMn, &tmB, fb, b_row + j * T::kAtomN,
                                                 kc * T::kBK, b);
                        }
                    } else {
                        if (hint)
                            tma_load_3d_pair_hint(b_dst, mapB, fb, kc * T::kBK, b_row, b, pol_b);
                        else
                            tma_load_3d_pair(b_dst, mapB, fb, kc * T::kBK, b_row, b);
                    }
                } else {
                    mbar_arrive_expect_tx(fb_local, tx);
#pragma unroll
                    for (int h = 0; h < T::kASub; ++h) {
                        if (hint)
                            tma_load_3d_hint(a_dst + h * T::kASubBytes, &tmA, fb_local, kc * T::kBK, a_row + h * kBM,
                                             b, pol_a);
                        else
                            tma_load_3d(a_dst + h * T::kASubBytes, &tmA, fb_local, kc * T::kBK, a_row + h * kBM, b);
                    }
                    if constexpr (kBMn) {
#pragma unroll 1
                        for (int j = 0; j < b_atoms; ++j) {
                            if (hint)
                                tma_load_3d_hint(b_dst + j * T::kBoxBytesMn, &tmB, fb_local,
                                                 b_row + j * T::kAtomN, kc * T::kBK, b, pol_b);
                            else
                                tma_load_3d(b_dst + j * T::kBoxBytesMn, &tmB, fb_local, b_row + j * T::kAtomN,
                                            kc * T::kBK, b);
                        }
                    } else {
                        if (hint)
                            tma_load_3d_hint(b_dst, mapB, fb_local, kc * T::kBK, b_row, b, pol_b);
                        else
                            tma_load_3d(b_dst, mapB, fb_local, kc * T::kBK, b_row, b);
                    }
                }
                issued |= 1u << stage;
                issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (aborted) break;
            if (leader) {  // the next work item
                if (p.sk) {
                    if (!sk_item(p, unit, ++sk_i, cur)) cur.t = -1;
                } else if (p.dynamic) {
                    int next = -1;
                    if (clc_pending) {
                        if (!wait_bounded(smem_u32(clcbar), clc_phase, abort_flag, p.timeout_ns,
                                          (blockIdx.x << 8) | 0x7Cu)) {
                            aborted = true;
                            break;
                        }
                        clc_pending = false;
                        clc_phase ^= 1u;
                        int first_cta;
                        if (clc_query(clc_resp, first_cta))
                            next = kPair ? first_cta / 2 : first_cta;
                        else
                            clc_live = false;  // nothing left to take over; never ask again
                    }
                    cur = WorkItem{next, 0, p.num_kb, kItemFull, unit};
                } else {
                    cur = WorkItem{t + units < num_work ? t + units : -1, 0, p.num_kb, kItemFull, unit};
                }
            }
        }
        // Tail: wait until every stage this CTA filled has been released, so
        // no MMA commit arrives on this CTA's barriers after it exits.
        for (int i = 0; i < kStages && !aborted; ++i) {
            if (!wait_bounded(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, p.timeout_ns,
                              (blockIdx.x << 8) | 0x50u | stage))
                break;
            if (++stage == kStages) {
                stage = 0;
                phase ^= 1u;
            }
        }
    } else if (threadIdx.x == 32 && leader) {
        // -------------------------------------------------- MMA issuer ----
        // int4 pairs: the second CTA's converter warps fill its half of each
        // stage and arrive (release, cluster scope) on these barriers
        constexpr bool kFullCluster = T::kI4 && kPair;
        int stage = 0;
        uint32_t phase = 0;
        bool aborted = false;
        int local = 0;
        for (;; ++local) {
            if (!wait_bounded(smem_u32(&qfull[q]), qph, abort_flag, p.timeout_ns, (blockIdx.x << 8) | 0x74u | q)) {
                aborted = true;
                break;
            }
            const WorkItem w = ring_get();
            ring_release();
            ring_next();
            const int t = w.t;
            if (t < 0) break;
            const int nkb = w.kb1 - w.kb0;            // k-blocks of this item
            const uint32_t idesc = t < p.split_from ? p.idesc : p.idesc_half;
            const int acc = local % T::kAccBufs;
            const uint32_t acc_phase = (local / T::kAccBufs) & 1;
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);  // wide: acc == 0
            // the MMAs of ring stage `st` (k-block kb) into accumulator half 0
            // (bit 0 of `halves`) and, for two-block shapes, half 1 (bit 1)
            const auto issue = [&](int st, int kb, int halves) {
                const uint32_t a_addr = stage0 + st * T::kStageBytes;
                const uint32_t b_addr = a_addr + T::kABytes;
#pragma unroll
                for (int k = 0; k < T::kKSteps; ++k) {
                    const uint64_t bdesc =
                        kBMn ? smem_desc_sw128(b_addr + k * T::kUmmaK * kBKBytes, T::kBoxBytesMn, 1024)
                             : smem_desc_sw128(b_addr + k * 32, 16, 1024);
                    const uint32_t accum = (kb | k) != 0 ? 1u : 0u;
#pragma unroll
                    for (int h = 0; h < T::kASub; ++h) {
                        if (!(halves & (1 << h))) continue;
                        const uint64_t adesc = smem_desc_sw128(a_addr + h * T::kASubBytes + k * 32, 16, 1024);
                        if constexpr (kPair)
                            umma_pair<kKind>(d_tmem + h * kBN, adesc, bdesc, idesc, accum);
                        else
                            umma<kKind>(d_tmem + h * kBN, adesc, bdesc, idesc, accum);
                    }
                }
            };
            const auto release_stage = [&]() {
                if constexpr (kPair)
                    umma_commit_pair(smem_u32(&empty[stage]), 0x3);
                else
                    umma_commit(smem_u32(&empty[stage]));
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            };
            // accumulator (half 0 for two-block shapes) released by the epilogue
            if (!wait_bounded(smem_u32(&tempty[acc]), acc_phase ^ 1u, abort_flag, p.timeout_ns,
                              (blockIdx.x << 8) | 0x20u | acc)) {
                aborted = true;
                break;
            }
            tc_fence_after();
            int kb0 = 0;
            if constexpr (kWide) {
                // Two-block shapes keep one tile in TMEM.  The epilogue frees
                // half 0 first; while half 1 is still being read, k-blocks go
                // into half 0 only (at most a ring-full: their stages stay
                // held), and once half 1 is free the same k-blocks go into it
                // (each half still accumulates in k order) and the tile
                // continues with both halves per stage.  A half 1 that is
                // already free (the first tile, or a drain that finished in
                // time) skips the detour.
                const int pre = nkb < kStages ? nkb : kStages;
                int st = stage;
                uint32_t ph = phase;
                int held = 0;  // k-blocks issued into half 0 only
                bool h1 = mbar_try_wait(smem_u32(&tempty[1]), acc_phase ^ 1u);
                while (!h1 && held < pre) {
                    if (!wait_bounded<kFullCluster>(smem_u32(&full[st]), ph, abort_flag, p.timeout_ns,
                                                    (blockIdx.x << 8) | 0x30u | st)) {
                        aborted = true;
                        break;
                    }
                    tc_fence_after();
                    issue(st, held, 1);
                    ++held;
                    if (++st == kStages) {
                        st = 0;
                        ph ^= 1u;
                    }
                    h1 = mbar_try_wait(smem_u32(&tempty[1]), acc_phase ^ 1u);
                }
                if (aborted) break;
                if (!h1 && !wait_bounded(smem_u32(&tempty[1]), acc_phase ^ 1u, abort_flag, p.timeout_ns,
                                         (blockIdx.x << 8) | 0x21u)) {
                    aborted = true;
                    break;
                }
                tc_fence_after();
                for (int kb = 0; kb < held; ++kb) {
                    issue(stage, kb, 2);
                    release_stage();
                }
                kb0 = held;
            }
            // two-block shapes: the last k-blocks (at most a ring-full) go
            // into half 0 first, so half 0 is complete -- and the epilogue
            // starts reading it -- while half 1 takes the same k-blocks
            const int last = kWide ? (nkb - kb0 < kStages ? nkb - kb0 : kStages) : 0;
            for (int kb = kb0; kb < nkb - last; ++kb) {
                if (!wait_bounded<kFullCluster>(smem_u32(&full[stage]), phase, abort_flag, p.timeout_ns,
                                                (blockIdx.x << 8) | 0x30u | stage)) {
                    aborted = true;
                    break;
                }
                tc_fence_after();
                issue(stage, kb, 3);
                release_stage();
            }
            if (aborted) break;
            if constexpr (kWide) {
                int st = stage;
                uint32_t ph = phase;
                for (int i = 0; i < last; ++i) {
                    if (!wait_bounded<kFullCluster>(smem_u32(&full[st]), ph, abort_flag, p.timeout_ns,
                                                    (blockIdx.x << 8) | 0x30u | st)) {
                        aborted = true;
                        break;
                    }
                    tc_fence_after();
                    issue(st, nkb - last + i, 1);
                    if (++st == kStages) {
                        st = 0;
                        ph ^= 1u;
                    }
                }
                if (aborted) break;
                if constexpr (kPair)
                    umma_commit_pair(smem_u32(&tfull[0]), 0x3);
                else
                    umma_commit(smem_u32(&tfull[0]));
                for (int i = 0; i < last; ++i) {
                    issue(stage, nkb - last + i, 2);
                    release_stage();
                }
                if constexpr (kPair)
                    umma_commit_pair(smem_u32(&tfull[1]), 0x3);
                else
                    umma_commit(smem_u32(&tfull[1]));
            } else {
                if constexpr (kPair)
                    umma_commit_pair(smem_u32(&tfull[acc]), 0x3);
                else
                    umma_commit(smem_u32(&tfull[acc]));
            }
        }
        // Tail: wait until both accumulators' last use has been released by
        // the epilogue(s), so no release arrives on this CTA after it exits.
        for (int i = 0; i < T::kAccBufs && !aborted; ++i, ++local) {
            const int acc = local % T::kAccBufs;
            if (!wait_bounded(smem_u32(&tempty[acc]), ((local / T::kAccBufs) & 1) ^ 1u, abort_flag, p.timeout_ns,
                              (blockIdx.x << 8) | 0x60u | acc))
                break;
            if constexpr (kWide) {  // and the second half
                if (!wait_bounded(smem_u32(&tempty[1]), (local & 1) ^ 1u, abort_flag, p.timeout_ns,
                                  (blockIdx.x << 8) | 0x61u))
                    break;
            }
        }
    } else if (warp >= 2 && warp < 6) {
        // ---------------------------------------------------- epilogue ----
        // Each warp owns 32 rows of the tile (its TMEM lane quarter) and
        // reads them 64 columns per tcgen05 wait (two 32x32b.x32 loads: lane
        // i gets row i).  With a tensor map for C (the usual case), every
        // 32 x 32 block goes out as one TMA store from a double-buffered,
        // swizzled staging tile, so the stores run asynchronously beside the
        // next loads.  Otherwise (peer destinations for the epilogue
        // all-gather, or C rows that are not 16-byte aligned) the block goes
        // through a staging tile with plain stores: 4 rows x 128 bytes per
        // instruction, to C and to every peer's C over NVLink.
        const int quarter = warp & 3;  // TMEM lanes this warp may read
        uint32_t* Cbits = static_cast<uint32_t*>(p.C);
        uint32_t* stile = epi_stage + (warp - 2) * 2 * 32 * 32;
        const uint32_t stile_s = smem_u32(stile);
        const uint32_t tempty_leader0 = kPair ? mapa_shared(smem_u32(&tempty[0]), 0) : smem_u32(&tempty[0]);
        const int rsub = lane >> 3;  // row within a 4-row group on the way out
        const int csub = lane & 7;   // 16-byte chunk (4 columns) within the 32 columns
        // dequantising epilogue: the per-tensor scales were produced on the
        // device by an earlier launch on the same stream
        const bool dequant = (kKind == kKindI8 || kKind == kKindI4) && p.scale_a != nullptr;
        const float combined = dequant ? __fmul_rn(*p.scale_a, *p.scale_b) : 0.f;
        uint32_t nstore = 0;  // TMA stores issued by this warp (selects the staging tile)
        const int flag_idx = static_cast<int>(rank) * 4 + quarter;  // stream-K flag of this warp's rows
        int local = 0;
        for (;; ++local) {
            if (!wait_bounded_warp<kPair>(smem_u32(&qfull[q]), qph, abort_flag, p.timeout_ns,
                                          (blockIdx.x << 8) | 0x7Au | q))
                break;
            const WorkItem w = ring_get();
            __syncwarp();
            if (lane == 0) ring_release();
            ring_next();
            const int t = w.t;
            if (t < 0) break;
            // stream-K: a head's C values are a partial sum that the tail's
            // epilogue adds to (TMA reduce-add) once the head has flagged them
            const bool head = w.kind == kItemHead, tail = w.kind == kItemTail;
            const int acc = local % T::kAccBufs;
            const uint32_t acc_phase = (local / T::kAccBufs) & 1;
            if (!wait_bounded_warp(smem_u32(&tfull[acc]), acc_phase, abort_flag, p.timeout_ns,
                                   (blockIdx.x << 8) | 0x40u | acc))
                break;
            tc_fence_after();
            if (tail) {
                // the head's stores of these rows are complete once its flag
                // carries this launch's tag (set long ago: heads run first)
                unsigned int* flag = sk_flag(p, w.unit - 1, flag_idx);
                uint64_t t0 = 0;
                bool seen = false;
                for (uint32_t i = 0;; ++i) {
                    seen = ld_acquire_gpu(flag) == p.sk_epoch;
                    if (__all_sync(0xffffffffu, seen)) break;
                    if (i == 0) t0 = global_timer_ns();
                    const bool stop = *abort_flag != 0u || global_timer_ns() - t0 > p.timeout_ns;
                    if (__any_sync(0xffffffffu, stop)) {
                        if (lane == 0 && *abort_flag == 0u)
                            record_failure(abort_flag, (blockIdx.x << 8) | 0xD0u | flag_idx);
                        break;
                    }
                }
                if (!__all_sync(0xffffffffu, seen)) break;
                if (lane == 0) {
                    *flag = 0u;                   // consumed: ready for a later launch
                    fence_proxy_async_global();   // the reduce-adds below come after the head's stores
                }
                __syncwarp();
            }
            int b, tm, tn, half;
            work_coords(t, p.split_from, p.tiles_m, p.tiles_n, p.group_m, b, tm, tn, half);
            const int col0 = tn * kBN + (half < 0 ? 0 : half * (kBN / 2));
            const int ncols = half < 0 ? kBN : kBN / 2;
            const long long cbase = static_cast<long long>(b) * p.batch_stride_c;
            bool lost = false;  // a bounded wait for half 1 gave up
#pragma unroll 1
            for (int h = 0; h < T::kASub; ++h) {  // wide tiles: the two 128-row halves
            if (kWide && h == 1) {
                // half 1 completes after half 0 (its last k-blocks are issued second)
                if (!wait_bounded_warp(smem_u32(&tfull[1]), acc_phase, abort_flag, p.timeout_ns,
                                       (blockIdx.x << 8) | 0x42u)) {
                    lost = true;
                    break;
                }
                tc_fence_after();
            }
            const int row0 =
                tm * T::kTileM + static_cast<int>(rank) * (T::kASub * kBM) + h * kBM + quarter * 32;
            const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                    static_cast<uint32_t>((acc + h) * kBN);
            if (p.tma_store) {
#pragma unroll 1
                for (int c = 0; c < ncols && row0 < p.M; c += 64) {  // (row0: warp-uniform)
                    const int col = col0 + c;
                    if (col >= p.N) break;  // warp-uniform
                    uint32_t va[32], vb[32];
                    tmem_ld_32x32b_x32(t_addr + c, va);
                    tmem_ld_32x32b_x32(t_addr + c + 32, vb);
                    tmem_ld_wait();
                    epi_convert<kAccF16, T::kI4>(va, dequant, combined);
                    epi_convert<kAccF16, T::kI4>(vb, dequant, combined);
                    epi_store_tma(&tmC, stile + (nstore & 1u) * 1024, stile_s + (nstore & 1u) * 4096, va, lane,
                                  col, row0, b, tail);
                    if (p.n_extra > 0) epi_store_peers(p, stile + (nstore & 1u) * 1024, row0, col, cbase, lane);
                    ++nstore;
                    if (c + 32 < ncols && col + 32 < p.N) {
                        epi_store_tma(&tmC, stile + (nstore & 1u) * 1024, stile_s + (nstore & 1u) * 4096, vb,
                                      lane, col + 32, row0, b, tail);
                        if (p.n_extra > 0)
                            epi_store_peers(p, stile + (nstore & 1u) * 1024, row0, col + 32, cbase, lane);
                        ++nstore;
                    }
                }
            } else {
#pragma unroll 1
            for (int c = 0; c < ncols; c += 32) {
                const int col = col0 + c;
                if (col >= p.N) break;  // warp-uniform
                uint32_t v[32];
                tmem_ld_32x32b_x32(t_addr + c, v);
                tmem_ld_wait();
                epi_convert<kAccF16, T::kI4>(v, dequant, combined);
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    *reinterpret_cast<uint4*>(stile + lane * 32 + ((q ^ (lane & 7)) << 2)) =
                        make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                __syncwarp();
                const int gcol = col + csub * 4;
#pragma unroll 2
                for (int it = 0; it < 8; ++it) {
                    const int r = it * 4 + rsub;
                    const uint4 w = *reinterpret_cast<const uint4*>(stile + r * 32 + ((csub ^ (r & 7)) << 2));
                    const int grow = row0 + r;
                    if (grow < p.M && gcol < p.N) {
                        const long long off = cbase + static_cast<long long>(grow) * p.N + gcol;
#pragma unroll 1
                        for (int d = -1; d < p.n_extra; ++d) {
                            uint32_t* dst = (d < 0 ? Cbits : static_cast<uint32_t*>(p.extra[d])) + off;
                            if (p.vec_store && gcol + 4 <= p.N) {
                                *reinterpret_cast<uint4*>(dst) = w;
                            } else {
                                dst[0] = w.x;
                                if (gcol + 1 < p.N) dst[1] = w.y;
                                if (gcol + 2 < p.N) dst[2] = w.z;
                                if (gcol + 3 < p.N) dst[3] = w.w;
                            }
                        }
                    }
                }
                __syncwarp();  // the tile is rewritten by the next 32 columns
            }
            }
            if constexpr (kWide) {
                // two-block shapes release each accumulator half as soon as
                // it is read: the next tile's MMAs start on half 0 meanwhile
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    const uint32_t tb = tempty_leader0 + static_cast<uint32_t>(h * sizeof(uint64_t));
                    if constexpr (kPair)
                        mbar_arrive_cluster(tb);
                    else
                        mbar_arrive(tb);
                }
            }
            }
            if (lost) break;
            if (head) {
                // the partial is in C once this warp's stores have completed:
                // flag it for the unit that finishes the tile
                if (lane == 0) {
                    bulk_wait_group_all();
                    fence_proxy_async_global();
                    __threadfence();
                    st_release_gpu(sk_flag(p, w.unit, flag_idx), p.sk_epoch);
                }
                __syncwarp();
            }
            if constexpr (!kWide) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    const uint32_t tb = tempty_leader0 + static_cast<uint32_t>(acc * sizeof(uint64_t));
                    if constexpr (kPair)
                        mbar_arrive_cluster(tb);
                    else
                        mbar_arrive(tb);
                }
            }
        }
        // the staging tiles are read before the CTA exits (and its shared
        // memory with them); the writes to C complete with the grid
        if (lane == 0 && nstore) bulk_wait_group_read<0>();
        __syncwarp();
    } else if (T::kI4 && warp >= 6) {
        // --------------------------------------------- int4 converters ----
        // Per k-block: wait for the stage's packed rows (this CTA's TMA, issued
        // once the MMAs had released the stage), widen them in place, make
        // the writes visible to the tensor core (async proxy), then report the
        // int8 stage filled on the leader's barrier, which the MMA issuer
        // waits on: the leader's converter warps arrive on it; a pair's second
        // CTA, once all its converter warps are done (named barrier 2), sends
        // one 16-byte copy into the leader's shared memory that completes on
        // it -- a remote arrive with cluster-scope release would stall each
        // warp for about a microsecond.  Every wait outcome goes through a
        // barrier-AND of the converter warps (named barrier 1), so they give
        // up together and none is left waiting at a barrier.
        constexpr int kConv = 32 * T::kConvWarps;
        using Plan = ConvPlan<kConv, T::kConvRows>;
        const int ct = (warp - 6) * 32 + lane;  // 0 .. kConv - 1
        const uint32_t full_leader0 = kPair ? mapa_shared(smem_u32(&full[0]), 0) : smem_u32(&full[0]);
        int ss = 0;
        uint32_t sph = 0;
        for (;;) {
            const bool got = wait_bounded_warp<kPair>(smem_u32(&qfull[q]), qph, abort_flag, p.timeout_ns,
                                                      (blockIdx.x << 8) | 0x7Bu);
            if (!named_barrier_and(1, kConv, got)) break;
            const WorkItem w = ring_get();
            __syncwarp();
            if (lane == 0) ring_release();
            ring_next();
            if (w.t < 0) break;
            int b, tm, tn, half;
            work_coords(w.t, p.split_from, p.tiles_m, p.tiles_n, p.group_m, b, tm, tn, half);
            const int rows = T::kASub * kBM + (half < 0 ? T::kBRows : T::kBRows / 2);
            bool ok = true;
            for (int kb = w.kb0; kb < w.kb1; ++kb) {
                uint8_t* stage_ptr = smem + ss * T::kStageBytes;
                const bool landed = wait_bounded_warp(smem_u32(&full_pk[ss]), sph, abort_flag, p.timeout_ns,
                                                      (blockIdx.x << 8) | 0xA0u | ss);
                uint4 v[Plan::kPasses];
                if (landed) conv_load<kConv, T::kConvRows>(stage_ptr + T::kPkOffset, rows, ct, v);
                if (!named_barrier_and(1, kConv, landed)) {  // every packed byte read (or all give up)
                    ok = false;
                    break;
                }
                conv_store<kConv, T::kConvRows>(stage_ptr, rows, ct, v);
                fence_proxy_async_smem();
                const uint32_t fb = full_leader0 + static_cast<uint32_t>(ss * sizeof(uint64_t));
                if (kPair && !leader) {
                    named_barrier_and(2, kConv, true);  // every converter warp's stores fenced
                    if (ct == 0) {
                        bulk_copy_to_cluster(mapa_shared(sig_buf, 0), sig_buf, T::kSignalBytes, fb);
                        signalled = true;
                    }
                } else {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(fb);
                }
                if (++ss == kStages) {
                    ss = 0;
                    sph ^= 1u;
                }
            }
            if (!ok) break;
        }
    }

    if (p.n_extra > 0) __threadfence_system();  // peer stores performed before the kernel ends
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (*abort_flag) {
        // Some role gave up.  Before shared and tensor memory are released,
        // let this CTA's own TMA copies land and its MMAs retire.
        if (threadIdx.x == 0 && issued) {
            if constexpr (T::kI4) {  // packed loads complete on this CTA's own barriers
                for (int s = 0; s < T::kPkStages; ++s)
                    if (issued & (1u << s)) drain_wait(smem_u32(&full_pk[s]), (issued_parity >> s) & 1u);
            } else if (!kPair || leader) {
                for (int s = 0; s < kStages; ++s)
                    if (issued & (1u << s)) drain_wait(smem_u32(&full[s]), (issued_parity >> s) & 1u);
            } else {
                // the peer's copies complete on the leader's barriers: give
                // them a fixed 2 ms, far above a copy's latency
                const uint64_t t0 = global_timer_ns();
                while (global_timer_ns() - t0 < 2000000ull) {
                }
            }
        }
        if (threadIdx.x == 0 && clc_pending) drain_wait(smem_u32(clcbar), clc_phase);  // response in flight
        if (signalled) {
            // a signal copy may still be reading this CTA's shared memory: give
            // it a fixed 2 ms, far above a copy's latency
            const uint64_t t0 = global_timer_ns();
            while (global_timer_ns() - t0 < 2000000ull) {
            }
        }
        if (threadIdx.x == 32 && leader) {
            if constexpr (kPair)
                umma_commit_pair_local(smem_u32(drain));
            else
                umma_commit(smem_u32(drain));
            drain_wait(smem_u32(drain), 0);
        }
        __syncwarp();
        __syncthreads();
    }
    if constexpr (kPair) cluster_sync_all();  // neither CTA frees TMEM / exits before the other is done
    tc_fence_after();
    if (warp == 1) {
        if constexpr (kPair)
            tmem_dealloc_pair(tmem_base, T::kTmemCols);
        else
            tmem_dealloc(tmem_base, T::kTmemCols);
    }
}

// Self-test of the bounded waits the GEMM uses: thread 0 (wait_bounded) and
// warp 1 (wait_bounded_warp) wait on an mbarrier nothing ever arrives on.
// Each wait gives up after timeout_ns and records the failure word; the
// kernel then returns normally, leaving the context usable.
__global__ void wait_selftest_kernel(unsigned long long timeout_ns)
{
    __shared__ uint64_t bar;
    __shared__ uint32_t flag;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        flag = 0u;
        fence_mbar_init();
    }
    __syncthreads();
    volatile uint32_t* abort_flag = &flag;
    if (threadIdx.x == 0) {
        wait_bounded(smem_u32(&bar), 0, abort_flag, timeout_ns, 0xFFu);
    } else if (threadIdx.x >= 32 && threadIdx.x < 64) {
        // returns once thread 0 has raised the flag (or on its own expiry)
        wait_bounded_warp(smem_u32(&bar), 0, abort_flag, timeout_ns, 0xFEu);
    }
    __syncthreads();
}

// Two tensors (A and B of an int4 GEMM) in one launch: 16-byte chunks
// [0, n0) of segment 0 then [0, n1) of segment 1, two chunks per thread per
// step; each segment's last n % 16 bytes (tail0, tail1) by block 0.
struct UnpackSeg {
    const uint4* in;
    uint4* out;
    long long n16;
    const int8_t* tail_in;
    int8_t* tail_out;
    int tail;
};

__device__ __forceinline__ uint4 unpack_load(const UnpackSeg& s0, const UnpackSeg& s1, long long i)
{
    return i < s0.n16 ? s0.in[i] : s1.in[i - s0.n16];
}

__device__ __forceinline__ void unpack_store(const UnpackSeg& s0, const UnpackSeg& s1, long long i, uint4 v)
{
    uint4 a, b;
    widen_word(v.x, a.x, a.y);
    widen_word(v.y, a.z, a.w);
    widen_word(v.z, b.x, b.y);
    widen_word(v.w, b.z, b.w);
    uint4* out = i < s0.n16 ? s0.out + 2 * i : s1.out + 2 * (i - s0.n16);
    out[0] = a;
    out[1] = b;
}

// Four chunks per thread per step, all four loads issued before any store.
__global__ void unpack_s4_kernel(const UnpackSeg s0, const UnpackSeg s1)
{
    grid_dependency_wait();
    grid_launch_dependents();
    const long long total = s0.n16 + s1.n16;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < total; i += 4 * stride) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = unpack_load(s0, s1, i + u * stride);
#pragma unroll
        for (int u = 0; u < 4; ++u) unpack_store(s0, s1, i + u * stride, v[u]);
    }
    for (; i < total; i += stride) unpack_store(s0, s1, i, unpack_load(s0, s1, i));
    if (blockIdx.x == 0) {
        const UnpackSeg& s = threadIdx.x < 16 ? s0 : s1;
        const int k = threadIdx.x & 15;
        if (threadIdx.x < 32 && k < s.tail) {
            const int8_t x = s.tail_in[k];
            s.tail_out[2 * k] = static_cast<int8_t>(static_cast<int8_t>(x << 4) >> 4);
            s.tail_out[2 * k + 1] = static_cast<int8_t>(x >> 4);
        }
    }
}

}  // namespace tcg
