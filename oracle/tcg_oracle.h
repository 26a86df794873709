/*
 * tcg_oracle.h -- CPU oracle for the tensor-core GEMM path (TEST INFRASTRUCTURE).
 *
 * This is the checker, never the product: only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / reference legs may load it.  The product path
 * (tensorcoreptx_b200, libtcgemm.so) never calls into it and has no CPU
 * fallback.
 *
 * Every function restates one function of the reference's host code
 * (MattJBorowski1991/TensorCorePTX, src/data*.cu) in plain C; each cites the
 * reference file:line it follows.  Parity is pinned two ways:
 *   - against the reference's own known answers printed in its committed
 *     Nsight logs (int8 C[0][0] = -149768, int4 C[0][0] = -563 at 512^3,
 *     seed 42; quant round-trip scales), see tests/test_oracle.py;
 *   - against the reference's own src/data*.cu compiled from source into
 *     oracle/_ref/ (oracle/Makefile, target `ref`), compared element by
 *     element on the same inputs.
 *
 * fp16 values are passed as raw IEEE binary16 bit patterns (uint16_t).
 */
#ifndef TCG_ORACLE_H
#define TCG_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- binary16 <-> binary32 (IEEE 754 round-to-nearest-even) ------------- */
uint16_t oracle_f32_to_f16(float x);
float    oracle_f16_to_f32(uint16_t h);

/* ---- reference-compatible seeded generators (glibc rand, srand(42)) ----- */
/* src/data.cu:6-14       */
void oracle_generate_fp16(uint16_t* A, uint16_t* B, int M, int N, int K, int batches);
/* src/data_int8.cu:6-14  */
void oracle_generate_int8(int8_t* A, int8_t* BT, int M, int N, int K, int batches);
/* src/data_int4.cu:26-42 */
void oracle_generate_int4_packed(int8_t* A, int8_t* BT, int M, int N, int K, int batches);
/* src/data_int8.cu:64-72 and src/data_int4.cu:94-100 (srand(43), Box-Muller
 * draws of src/data_int8.cu:56-60) */
void oracle_generate_fp32_normal(float* A, float* BT, int M, int N, int K, int batches);

/* ---- GEMMs (one batch; row range [row0, row0+rows) of C) ---------------- */
/* src/data.cu:16-24: f32 accumulate in k order, B is K x N row-major        */
void oracle_gemm_f16_f32acc(const uint16_t* A, const uint16_t* B, float* C,
                            int M, int N, int K, int row0, int rows);
/* fp64 accumulate (the fp16 tolerance anchor); b_kn != 0: B is K x N
 * row-major, else B is given transposed (N x K row-major).                  */
void oracle_gemm_f16_f64(const uint16_t* A, const uint16_t* B, double* C,
                         int M, int N, int K, int b_kn, int row0, int rows);
/* src/data_int8.cu:18-26: exact int32, B given as BT (N x K)               */
void oracle_gemm_s8(const int8_t* A, const int8_t* BT, int32_t* C,
                    int M, int N, int K, int row0, int rows);
/* same product with B as K x N row-major                                    */
void oracle_gemm_s8_kn(const int8_t* A, const int8_t* B, int32_t* C,
                       int M, int N, int K, int row0, int rows);
/* src/data_int4.cu:46-61: packed nibbles, low nibble = even k              */
void oracle_gemm_s4(const int8_t* Ap, const int8_t* BTp, int32_t* C,
                    int M, int N, int K, int row0, int rows);
/* src/data_int8.cu:97-105: fp64 accumulate, B given as BT                   */
void oracle_gemm_f32(const float* A, const float* BT, float* C,
                     int M, int N, int K, int row0, int rows);

/* fp8 (OCP FP8: e4m3 = bias 7, no infinities, S.1111.111 is NaN;
 * e5m2 = bias 15, IEEE-style inf/NaN) -> float, exact.  fmt 0 = e4m3, 1 = e5m2.
 * The reference has no fp8 path; this anchors the fp8 GEMM (its tolerance is
 * the fp16 one, against this fp64 product). */
double oracle_f8_to_f64(uint8_t v, int fmt);
void oracle_gemm_f8_f64(const uint8_t* A, const uint8_t* B, double* C, int M, int N, int K,
                        int a_fmt, int b_fmt, int b_kn, int row0, int rows);

/* ---- nibble helpers (src/data_int4.cu:10-22) ----------------------------- */
void oracle_unpack_s4(const int8_t* packed, int8_t* out, long n_packed_bytes);

/* ---- quantisation path --------------------------------------------------- */
/* src/data_int8.cu:74-89 */
float oracle_quantize_absmax_s8(const float* src, int8_t* dst, long n);
/* src/data_int4.cu:104-127 */
float oracle_quantize_absmax_s4(const float* src, int8_t* dst_packed, int rows, int cols_k);
/* src/data_int8.cu:91-95 */
void oracle_dequantize(const int32_t* src, float* dst, long n, float scale_a, float scale_bt);

/* ---- accuracy metrics ---------------------------------------------------- */
typedef struct { float max_abs_err, rmse, real_err_pct; int pass; } oracle_acc_f32;
typedef struct { int32_t max_abs_err; float rmse; int max_row, max_col;
                 int32_t ref_at_max, out_at_max; int pass; } oracle_acc_i32;
typedef struct { float max_abs_err, rmse, real_err_pct, snr_db; int pass; } oracle_acc_quant;

/* src/data.cu:38-52 */
oracle_acc_f32 oracle_measure_accuracy(const float* ref, const float* out, int M, int N, float pass_tol);
/* src/data_int8.cu:28-50 (identical to src/data_int4.cu:65-84) */
oracle_acc_i32 oracle_measure_accuracy_i32(const int32_t* ref, const int32_t* out, int M, int N);
/* src/data_int8.cu:107-125 */
oracle_acc_quant oracle_measure_accuracy_quant(const float* ref, const float* out, int M, int N, float pass_tol);

#ifdef __cplusplus
}
#endif
#endif
