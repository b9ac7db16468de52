// Tensor-core GEMM (tcgen05 + TMA, sm_100a) and related internal entry points.
#pragma once
#include <cuda.h>

#include "lc_common.cuh"

// What the GEMM epilogue does with the f32 accumulator tile before the store.
enum GemmEpiKind : int {
  EPI_PLAIN = 0,     // y = acc (+ bias[n])
  EPI_RESIDUAL = 1,  // y = acc + resid[m, n]            (attention / MLP output projections)
  EPI_ROPE_QKV = 2,  // q,k columns rotated by RoPE at pos[m] (fused Wqkv projection)
  EPI_GEGLU = 3,     // y[m, j] = gelu(acc[m, v(j)]) * acc[m, g(j)] with value/gate interleaved in 32-column blocks
};

struct GemmEpilogue {
  int kind = EPI_PLAIN;
  const void* resid = nullptr;      // EPI_RESIDUAL: [M, N] in the output dtype, row stride ldr
  int64_t ldr = 0;
  const int32_t* pos = nullptr;     // EPI_ROPE_QKV: position of each row
  const float* rope_cs = nullptr;   // EPI_ROPE_QKV: cos/sin table [32][cap] ++ [32][cap] (position-minor)
  int rope_cap = 0;
  int rope_cols = 0;                // EPI_ROPE_QKV: columns [0, rope_cols) are rotated (q and k), head dim 64
};

namespace lc {
// y[M, N] = x[M, K] · w[N, K]ᵀ (+ bias) with the tcgen05 kernel. Returns false
// (and does nothing) when the shapes/dtypes/alignment do not fit the kernel.
bool gemm_linear(const LcTensor* x2, const LcTensor* w, const LcTensor* bias, LcTensor* y, const GemmEpilogue& ep);
// Raw-pointer form used by the fused encoder: all dense row-major, dtype f16/bf16.
bool gemm_raw(const void* x, int64_t M, int64_t K, const void* w, int64_t N, const void* bias, int bias_dtype, void* y, int64_t ldy,
              int dtype, const GemmEpilogue& ep, cudaStream_t st);
void linear_simt(const LcTensor* x2, const LcTensor* w, const LcTensor* bias, LcTensor* y);
const float* rope_table(int D, double base, int L, int* cap_out, bool position_minor = false);
bool attention_try_fast(const LcTensor* q, const LcTensor* k, const LcTensor* v, const LcTensor* m, float scale, LcTensor* y);
// Reads and clears the device-side error words of the pipelined kernels.
std::string take_device_errors();
std::string take_attention_errors();
// Cached 2-D tiled tensor map (128-byte swizzle) over a row-major [rows, cols] matrix with row stride ld.
const CUtensorMap& tensor_map_2d(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_cols, int box_rows, int dtype);
// tcgen05 varlen attention (lc_attention_tc.cu) and its 128-row tile list.
std::vector<int4> attention_tiles_tc(const int32_t* cu, int nseq);
void attention_varlen_tc(const void* qkv, void* out, const int4* tiles_dev, int ntiles, int64_t T, int H, int half_window, float scale,
                         int dtype, cudaStream_t st);
}  // namespace lc
void lc_gemm_destroy_caches();
