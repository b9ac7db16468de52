// Tensor-core GEMM (tcgen05 + TMA, sm_100a) and related internal entry points.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>

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
  const float* rope_cs = nullptr;   // EPI_ROPE_QKV: table [16][cap] of float4 (cos 2i, cos 2i+1, sin 2i, sin 2i+1)
  int rope_cap = 0;
  int rope_cols = 0;                // EPI_ROPE_QKV: columns [0, rope_cols) are rotated (q and k), head dim 64
  // LayerNorm folded into the next projection (the fused encoder): a residual
  // GEMM records row statistics of what it stores, and the projection that
  // consumes LayerNorm(y)·diag(γ) turns x·(W·diag(γ))ᵀ into the normalised
  // product: out = r·(acc − μ·wsum[n]) with μ, r = 1/sqrt(var + eps) of row m.
  float2* stats_out = nullptr;       // EPI_RESIDUAL: (mean, M2) of the stored row per gemm_stats_part_cols(N) columns
  const float2* ln_stats = nullptr;  // the statistics to apply: [M][ln_parts], ln_part_cols columns per part
  const float* ln_wsum = nullptr;    // Σ_k W[n, k]·γ[k] per accumulator column n (16-byte aligned)
  int ln_parts = 0, ln_part_cols = 0, ln_cols = 0;
  float ln_eps = 0.f;
  // The weight is not written by any kernel of the current launch chain (a
  // resident dense weight, not a dequantisation scratch): the kernel may
  // request it before waiting for its predecessor.
  bool w_static = false;
  // The weight of the next projection of the chain (or null): the CTAs bring
  // it into L2 while this one runs, so the next GEMM's weight blocks come from
  // L2 rather than HBM (few rows: the chain is latency-bound). 16-byte aligned.
  const void* l2_next = nullptr;
  size_t l2_next_bytes = 0;
};

// A weight in the native packed 4/8-bit layout (packages/tensor-backend/src/index.ts:98-108)
// for gemm_raw_q: rows of K·bits/8 bytes, scales / biases [N, ceil(K/g)].
struct GemmQuantB {
  const uint8_t* w = nullptr;
  const void* scales = nullptr;
  const void* biases = nullptr;  // null for symmetric weights
  int sdt = 0, bits = 0, group = 0, mode = 0;
  const float* gamma = nullptr;  // optional column scale [K] (a folded LayerNorm weight)
};

namespace lc {
// y[M, N] = x[M, K] · w[N, K]ᵀ (+ bias) with the tcgen05 kernel. Returns false
// (and does nothing) when the shapes/dtypes/alignment do not fit the kernel.
bool gemm_linear(const LcTensor* x2, const LcTensor* w, const LcTensor* bias, LcTensor* y, const GemmEpilogue& ep);
// Raw-pointer form used by the fused encoder: all dense row-major, dtype f16/bf16.
bool gemm_raw(const void* x, int64_t M, int64_t K, const void* w, int64_t N, const void* bias, int bias_dtype, void* y, int64_t ldy,
              int dtype, const GemmEpilogue& ep, cudaStream_t st);
// The same product with the weight dequantised inside the GEMM (the packed
// tile is loaded by TMA and turned into the MMA's 16-bit operand in shared
// memory, bit-identical to dequantising into a dense matrix first). Taken for
// few rows (one prompt, small batches), where the weight stream dominates;
// returns false (nothing launched) otherwise.
bool gemm_raw_q(const void* x, int64_t M, int64_t K, const GemmQuantB& q, int64_t N, const void* bias, int bias_dtype, void* y,
                int64_t ldy, int dtype, const GemmEpilogue& ep, cudaStream_t st);
// N-tile width gemm_raw uses for an accumulator of Nacc columns.
int gemm_tile_n(int64_t Nacc, bool geglu);
// Row statistics of a residual GEMM (GemmEpilogue::stats_out) come in parts of
// this many columns: [M][ceil(N / part)].
int gemm_stats_part_cols(int64_t N);
void linear_simt(const LcTensor* x2, const LcTensor* w, const LcTensor* bias, LcTensor* y);
const float* rope_table(int D, double base, int L, int* cap_out, bool position_minor = false);
// The contract's sdpa on tensor cores (lc_attention.cu) when q/k/v/y suit it;
// false, with nothing launched, otherwise.
bool sdpa_flash(const LcTensor* q, const LcTensor* k, const LcTensor* v, const LcTensor* m, float scale, LcTensor* y);
// Reads and clears the device-side error words of the pipelined kernels.
std::string take_device_errors();
std::string take_attention_errors();
// Cached 2-D tiled tensor map (128-byte swizzle) over a row-major [rows, cols] matrix with row stride ld.
CUtensorMap tensor_map_2d(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_cols, int box_rows, int dtype);
// The driver's cuTensorMapEncodeTiled (for maps of other ranks than tensor_map_2d's).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();
// The contract's sdpa on the tcgen05 attention kernel (lc_attention_tc.cu) for
// f16/bf16 head dim 64 with 16-byte strides; *out is a new [B, nh, Lq, 64]
// view. False, with nothing launched, otherwise.
bool sdpa_tc(const LcTensor* q, const LcTensor* k, const LcTensor* v, const LcTensor* m, float scale, LcTensor** out);
// tcgen05 varlen attention (lc_attention_tc.cu) and its 128-row tile list.
std::vector<int4> attention_tiles_tc(const int32_t* cu, int nseq);
void attention_varlen_tc(const void* qkv, void* out, const int4* tiles_dev, int ntiles, int64_t T, int H, int half_window, float scale,
                         int dtype, cudaStream_t st);
}  // namespace lc
void lc_gemm_destroy_caches();
