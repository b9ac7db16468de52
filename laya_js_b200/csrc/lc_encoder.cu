// Fused ModernBERT encoder over packed variable-length sequences.
//
// Computes ModernBert.encode (packages/modernbert/src/index.ts:407-429) for
// every valid token, layer by layer as ModernBert.layer (index.ts:342-357)
// does, with these fusions:
//   embedding + LayerNorm                          -> k_embed_ln
//   Wqkv linear + reshape/transpose/split + RoPE   -> GEMM, EPI_ROPE_QKV (q/k rotated at each token's position)
//   masks + sdpa + transpose/reshape               -> attention_varlen (window rule in-kernel)
//   Wo linear + residual add                       -> GEMM, EPI_RESIDUAL (in place on x)
//   mlp_norm + Wi linear + geglu                   -> GEMM, EPI_GEGLU (Wi rows interleaved in 32-row blocks at load)
//   mlp.Wo linear + residual add                   -> GEMM, EPI_RESIDUAL (in place on x)
//   attn_norm (layers >= 1) + Wqkv                 -> the EPI_ROPE_QKV GEMM
// The two LayerNorms of a layer are folded into the projection after them:
// LayerNorm(x)·Wᵀ = r·(x·(W·diag(γ))ᵀ − μ·Σ_k W[n,k]γ[k]) per row, with μ and
// r = 1/sqrt(var + eps) from row statistics the residual GEMM before records
// in its epilogue; no normalised copy of the hidden states is written.
// plus the CLS classifier head + softmax (packages/laya/src/model.ts:228 pattern).
// Quantized Linear weights (4/8-bit, laya-js packing) stay packed in HBM and
// are dequantised per GEMM into one reusable f16/bf16 scratch matrix.
#include "lc_api.h"
#include "lc_gemm.h"
#include "lc_quant.cuh"
#include "lc_sm100.cuh"
#include "laya_cuda_encoder.h"

#include <algorithm>
#include <memory>
#include <unordered_set>

using namespace lc;

namespace lc {
void layernorm_raw(const void* x, const float* w, void* y, int64_t rows, int N, float eps, int dtype, cudaStream_t st);
void copy_into(const LcTensor* src, LcTensor* dst_dense);
std::vector<int4> attention_tiles(const int32_t* cu, int nseq);
void attention_varlen(const void* qkv, void* out, const int4* tiles_dev, int ntiles, int64_t T, int H, int half_window, float scale,
                      int dtype, cudaStream_t st);
void dequant_into(const LcTensor* w, const LcTensor* s, const LcTensor* b, int bits, int g, int mode, LcTensor* out);
void dequant_scaled_into(const LcTensor* w, const LcTensor* s, const LcTensor* b, int bits, int g, int mode, const float* gamma, LcTensor* out);
}  // namespace lc

namespace {

__global__ void k_positions(const int32_t* __restrict__ cu, int nseq, int32_t* __restrict__ pos) {
  pdl_trigger();
  pdl_wait();
  for (int s = blockIdx.x; s < nseq; s += gridDim.x) {
    int a = cu[s], b = cu[s + 1];
    for (int t = a + threadIdx.x; t < b; t += blockDim.x) pos[t] = t - a;
  }
}

// x[t] = LayerNorm(table[ids[t]]) * w, one warp per token, H <= 2048, H % 8 == 0
template <typename T, int MAXV>
__global__ void __launch_bounds__(256) k_embed_ln(const T* __restrict__ table, int64_t V, const int32_t* __restrict__ ids,
                                                  const float* __restrict__ w, T* __restrict__ y, int64_t rows, int H, float eps) {
  pdl_trigger();
  pdl_wait();
  int lane = threadIdx.x & 31;
  int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int nv = H / 8;
  for (int64_t r = warp; r < rows; r += nwarps) {
    int64_t id = ids[r];
    if (id < 0 || id >= V) id = 0;  // out-of-range ids read row 0 (never fault)
    const T* src = table + id * H;
    float v[MAXV][8];
    float s = 0.f;
#pragma unroll
    for (int t = 0; t < MAXV; t++) {
      int c = t * 32 + lane;
      if (c < nv) {
        uint4 raw = *(const uint4*)(src + c * 8);
        const T* e = (const T*)&raw;
#pragma unroll
        for (int j = 0; j < 8; j++) {
          float f = std::is_same<T, __half>::value ? __half2float(((const __half*)e)[j]) : __bfloat162float(((const __nv_bfloat16*)e)[j]);
          v[t][j] = f;
          s += f;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    float mu = s / H, q = 0.f;
#pragma unroll
    for (int t = 0; t < MAXV; t++)
      if (t * 32 + lane < nv)
#pragma unroll
        for (int j = 0; j < 8; j++) q += (v[t][j] - mu) * (v[t][j] - mu);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    float rs = rsqrtf(q / H + eps);
#pragma unroll
    for (int t = 0; t < MAXV; t++) {
      int c = t * 32 + lane;
      if (c < nv) {
        uint4 raw;
        T* e = (T*)&raw;
#pragma unroll
        for (int j = 0; j < 8; j++) {
          float o = (v[t][j] - mu) * rs * __ldg(w + c * 8 + j);
          if constexpr (std::is_same<T, __half>::value) e[j] = __float2half_rn(o);
          else e[j] = __float2bfloat16_rn(o);
        }
        *(uint4*)(y + r * H + c * 8) = raw;
      }
    }
  }
}

// probs[s] = softmax(hidden[cu[s]] · Wᵀ + b), one block per sequence, f32 accumulation
template <typename T>
__global__ void k_cls_head(const T* __restrict__ hidden, int H, const int32_t* __restrict__ cu, int nseq, const char* w, int wdt,
                           const char* b, int bdt, int C, float* __restrict__ probs) {
  extern __shared__ float logits[];
  pdl_trigger();
  pdl_wait();
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int s = blockIdx.x; s < nseq; s += gridDim.x) {
    const T* row = hidden + (int64_t)cu[s] * H;
    for (int c = warp; c < C; c += nw) {
      float acc = 0.f;
      for (int k = lane; k < H; k += 32) acc += ld_as<float>((const char*)row, std::is_same<T, __half>::value ? LC_F16 : LC_BF16, k) * ld_as<float>(w, wdt, (int64_t)c * H + k);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) logits[c] = acc + (b ? ld_as<float>(b, bdt, c) : 0.f);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float m = -INFINITY;
      for (int c = 0; c < C; c++) m = fmaxf(m, logits[c]);
      float z = 0.f;
      for (int c = 0; c < C; c++) z += expf(logits[c] - m);
      for (int c = 0; c < C; c++) probs[(int64_t)s * C + c] = expf(logits[c] - m) / z;
    }
    __syncthreads();
  }
}

// LayerNorm weight folded into the projection that reads the norm's output:
// Wout[n, k] = round(W[n, k]·γ[k]) (Wout may be null) and wsum[n] = Σ_k of
// those rounded values, one warp per row.
template <typename T>
__global__ void k_fold_norm(const T* __restrict__ W, const float* __restrict__ gamma, T* __restrict__ Wout, float* __restrict__ wsum, int64_t N,
                            int64_t K) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t n = warp; n < N; n += nwarps) {
    double acc = 0.0;
    for (int64_t k = lane; k < K; k += 32) {
      const T v = sm100::TcFmt<T>::cvt(sm100::TcFmt<T>::back(W[n * K + k]) * gamma[k]);
      if (Wout) Wout[n * K + k] = v;
      acc += (double)sm100::TcFmt<T>::back(v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) wsum[n] = (float)acc;
  }
}

__global__ void k_permute_rows(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t rowbytes, const int32_t* __restrict__ perm,
                               int64_t rows) {
  LC_GRID_STRIDE(i, rows * rowbytes) {
    int64_t r = i / rowbytes, c = i % rowbytes;
    dst[i] = src[(int64_t)perm[r] * rowbytes + c];
  }
}

struct Mat {
  LcTensor* dense = nullptr;  // [N, K] in the compute dtype
  LcTensor* q = nullptr;      // packed [N, K*bits/8]
  LcTensor* s = nullptr;
  LcTensor* b = nullptr;
  int64_t N = 0, K = 0;
  // folded LayerNorm (the projection reads the norm's input): γ (f32 [K]) and
  // wsum (f32 [N]) = row sums of W·diag(γ); dense weights are stored folded
  const float* gamma = nullptr;
  LcTensor* wsum = nullptr;
};

struct Layer {
  int kind = 0;
  LcTensor* attn_norm = nullptr;
  LcTensor* mlp_norm = nullptr;
  Mat Wqkv, Wo, Wi, WoMlp;
};

struct Encoder {
  lc_encoder_config cfg{};
  std::vector<Layer> layers;
  LcTensor* tok = nullptr;
  LcTensor* emb_norm = nullptr;
  LcTensor* final_norm = nullptr;
  std::vector<LcTensor*> owned;  // references released by lc_encoder_free
  // workspace (grow-only)
  void* ws = nullptr;
  size_t ws_bytes = 0;
  LcTensor* deq = nullptr;  // dequant scratch for quantized weights
  // host staging (pinned) for cu_seqlens + tiles
  void* stage = nullptr;
  size_t stage_bytes = 0;
  cudaEvent_t stage_ev = nullptr;
  void* ids_stage = nullptr;
  size_t ids_stage_bytes = 0;
  void* probs_stage = nullptr;
  size_t probs_stage_bytes = 0;
  // tracing: CUDA events around each kernel class (0 GEMM, 1 attention, 2 LN/embedding, 3 head/other)
  bool prof = false;
  std::vector<cudaEvent_t> ev_pool;
  std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> pending;
  double prof_ms[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int64_t prof_n[8] = {0, 0, 0, 0, 0, 0, 0, 0};
};

cudaEvent_t pooled_event(Encoder* e) {
  if (!e->ev_pool.empty()) {
    cudaEvent_t ev = e->ev_pool.back();
    e->ev_pool.pop_back();
    return ev;
  }
  cudaEvent_t ev;
  CUDA_OK(cudaEventCreate(&ev));
  return ev;
}

// Records an event pair around the kernels issued in its lifetime when profiling is on.
struct Prof {
  Encoder* e;
  int cls;
  cudaEvent_t a = nullptr;
  Prof(Encoder* e_, int c) : e(e_), cls(c) {
    if (e->prof) {
      a = pooled_event(e);
      CUDA_OK(cudaEventRecord(a, stream()));
    }
  }
  ~Prof() {
    if (a) {
      cudaEvent_t b = pooled_event(e);
      cudaEventRecord(b, stream());
      e->pending.push_back({cls, {a, b}});
    }
  }
  // nothing was launched in this interval: drop it
  void cancel() {
    if (a) e->ev_pool.push_back(a);
    a = nullptr;
  }
};

std::unordered_set<Encoder*>& encoders() {
  static std::unordered_set<Encoder*> s;
  return s;
}

Encoder* check_enc(uint64_t h) {
  Encoder* e = reinterpret_cast<Encoder*>(h);
  LC_CHECK(h && encoders().count(e), "encoder: invalid or freed encoder handle");
  return e;
}

LcTensor* keep(Encoder* e, LcTensor* t) {
  LcTensor* v = view_of(t, t->dims(), std::vector<int64_t>(t->strides, t->strides + t->ndim), t->offset);
  e->owned.push_back(v);
  return v;
}

// A LayerNorm weight as an owned f32 copy (the norm kernels read f32 vectors).
LcTensor* keep_f32(Encoder* e, LcTensor* t) {
  LcTensor* f = alloc(LC_F32, {t->numel()});
  copy_into(t, f);
  e->owned.push_back(f);
  return f;
}

void need_shape(const LcTensor* t, std::vector<int64_t> want, const std::string& what) {
  LC_CHECK(t->dims() == want, "encoder: " + what + " has shape " + shape_str(t->dims()) + ", want " + shape_str(want));
  LC_CHECK(t->contiguous(), "encoder: " + what + " must be dense");
}

// GeGLU interleave: output rows [v 32 | g 32] per 32-row block of the two halves.
std::vector<int32_t> geglu_perm(int64_t I) {
  std::vector<int32_t> p;
  for (int64_t b = 0; b < I / 32; b++) {
    for (int j = 0; j < 32; j++) p.push_back((int32_t)(b * 32 + j));
    for (int j = 0; j < 32; j++) p.push_back((int32_t)(I + b * 32 + j));
  }
  return p;
}

LcTensor* permuted_rows(Encoder* e, const LcTensor* src, const std::vector<int32_t>& perm) {
  LcTensor* dst = alloc(src->dtype, src->dims());
  int32_t* d = (int32_t*)dmalloc(perm.size() * 4);
  CUDA_OK(cudaMemcpyAsync(d, perm.data(), perm.size() * 4, cudaMemcpyHostToDevice, stream()));
  int64_t rowbytes = src->numel() / src->shape[0] * dtype_size(src->dtype);
  k_permute_rows<<<blocks_for(src->shape[0] * rowbytes, 256), 256, 0, stream()>>>((const uint8_t*)src->data(), (uint8_t*)dst->data(), rowbytes,
                                                                                  d, src->shape[0]);
  LC_LAUNCHED(1);
  dfree(d);
  e->owned.push_back(dst);
  return dst;
}

Mat take_mat(Encoder* e, const lc_tensor* w, int& i, int64_t N, int64_t K, const std::string& what, bool geglu) {
  Mat m;
  m.N = N;
  m.K = K;
  const lc_encoder_config& c = e->cfg;
  if (c.quant_bits == 0) {
    LcTensor* t = check(w[i++], what.c_str());
    need_shape(t, {N, K}, what);
    LC_CHECK(t->dtype == c.dtype, "encoder: " + what + " must be stored in the encoder dtype");
    m.dense = geglu ? permuted_rows(e, t, geglu_perm(N / 2)) : keep(e, t);
  } else {
    LcTensor* q = check(w[i++], what.c_str());
    LcTensor* s = check(w[i++], what.c_str());
    LcTensor* b = w[i] ? check(w[i], what.c_str()) : nullptr;
    i++;
    int64_t G = (K + c.quant_group - 1) / c.quant_group;
    need_shape(q, {N, K * c.quant_bits / 8}, what + " (packed)");
    need_shape(s, {N, G}, what + " scales");
    if (c.quant_mode == 1) {
      LC_CHECK(b, "encoder: " + what + ": affine weights need biases");
      need_shape(b, {N, G}, what + " biases");
    }
    if (geglu) {
      auto p = geglu_perm(N / 2);
      m.q = permuted_rows(e, q, p);
      m.s = permuted_rows(e, s, p);
      m.b = b ? permuted_rows(e, b, p) : nullptr;
    } else {
      m.q = keep(e, q);
      m.s = keep(e, s);
      m.b = b ? keep(e, b) : nullptr;
    }
  }
  return m;
}

// Folds LayerNorm weight γ into the projection that consumes the norm's output
// (ModernBertLayer: Wqkv after attn_norm, Wi after mlp_norm): dense weights are
// replaced by W·diag(γ); packed weights stay packed and their per-forward
// dequantisation applies γ. wsum = row sums of the folded weight.
void fold_norm(Encoder* e, Mat& m, const LcTensor* gamma) {
  const lc_encoder_config& c = e->cfg;
  m.gamma = (const float*)gamma->data();
  m.wsum = alloc(LC_F32, {m.N});
  e->owned.push_back(m.wsum);
  LcTensor* src = m.dense;
  LcTensor* tmp = nullptr;
  if (!src) {
    tmp = alloc(c.dtype, {m.N, m.K});
    dequant_into(m.q, m.s, m.b, c.quant_bits, c.quant_group, c.quant_mode, tmp);
    src = tmp;
  }
  LcTensor* out = m.dense ? alloc(c.dtype, {m.N, m.K}) : nullptr;
  unsigned blocks = blocks_for(m.N * 32, 256);
  if (c.dtype == LC_F16)
    k_fold_norm<__half><<<blocks, 256, 0, stream()>>>((const __half*)src->data(), m.gamma, out ? (__half*)out->data() : nullptr,
                                                      (float*)m.wsum->data(), m.N, m.K);
  else
    k_fold_norm<__nv_bfloat16><<<blocks, 256, 0, stream()>>>((const __nv_bfloat16*)src->data(), m.gamma,
                                                             out ? (__nv_bfloat16*)out->data() : nullptr, (float*)m.wsum->data(), m.N, m.K);
  LC_LAUNCHED(1);
  if (tmp) release(tmp);
  if (out) {
    auto it = std::find(e->owned.begin(), e->owned.end(), m.dense);
    if (it != e->owned.end()) {
      e->owned.erase(it);
      release(m.dense);
    }
    m.dense = out;
    e->owned.push_back(out);
  }
}

// y = x · Wᵀ with the given epilogue (dense weight or packed weight dequantised into the scratch)
void run_gemm(Encoder* e, const Mat& m, const void* x, int64_t M, void* y, int64_t ldy, const GemmEpilogue& ep, int64_t n_out, int cls) {
  const void* w;
  if (m.dense) {
    w = m.dense->data();
  } else {
    // few rows: dequantise inside the GEMM (the weight stream dominates)
    GemmQuantB qb;
    qb.w = (const uint8_t*)m.q->data();
    qb.scales = m.s->data();
    qb.biases = m.b ? m.b->data() : nullptr;
    qb.sdt = m.s->dtype;
    qb.bits = e->cfg.quant_bits;
    qb.group = e->cfg.quant_group;
    qb.mode = e->cfg.quant_mode;
    qb.gamma = m.gamma;
    {
      Prof p(e, cls);
      if (gemm_raw_q(x, M, m.K, qb, n_out, nullptr, 0, y, ldy, e->cfg.dtype, ep, stream())) return;
      p.cancel();
    }
    if (!e->deq || e->deq->numel() < m.N * m.K) {
      if (e->deq) release(e->deq);
      int64_t biggest = 0;
      for (auto& l : e->layers)
        for (const Mat* mm : {&l.Wqkv, &l.Wo, &l.Wi, &l.WoMlp}) biggest = std::max(biggest, mm->N * mm->K);
      e->deq = alloc(e->cfg.dtype, {biggest});
    }
    LcTensor* view = view_of(e->deq, {m.N, m.K}, {m.K, 1}, 0);
    Prof pd(e, 3);
    if (m.gamma) dequant_scaled_into(m.q, m.s, m.b, e->cfg.quant_bits, e->cfg.quant_group, e->cfg.quant_mode, m.gamma, view);
    else dequant_into(m.q, m.s, m.b, e->cfg.quant_bits, e->cfg.quant_group, e->cfg.quant_mode, view);
    release(view);
    w = e->deq->data();
  }
  Prof p(e, cls);
  GemmEpilogue epw = ep;
  epw.w_static = m.dense != nullptr;  // the dequantisation scratch is written inside the chain
  bool ok = gemm_raw(x, M, m.K, w, n_out, nullptr, 0, y, ldy, e->cfg.dtype, epw, stream());
  LC_CHECK(ok, "encoder: the tcgen05 GEMM rejected a projection shape");
}

void grow_ws(Encoder* e, size_t bytes) {
  if (e->ws_bytes >= bytes) return;
  if (e->ws) dfree(e->ws);
  e->ws = dmalloc(bytes);
  e->ws_bytes = bytes;
}

void* grow_pinned(void*& p, size_t& have, size_t want) {
  if (have >= want) return p;
  if (p) CUDA_OK(cudaFreeHost(p));
  CUDA_OK(cudaHostAlloc(&p, want, cudaHostAllocDefault));
  have = want;
  return p;
}

void run_kernels(Encoder* e, char* ws, int64_t T, int nseq, int maxlen, const int32_t* cu_dev, const int4* tiles_dev, int ntiles,
                 const int32_t* ids_dev, void* hidden_out, const LcTensor* head_w, const LcTensor* head_b, float* probs_dev,
                 cudaStream_t st);

// Frees the CUDA graphs captured on an encoder (they reference its weights).
void free_graphs_of(Encoder* e);

// Workspace of one forward over T tokens: x [T,H] | h [T,H] | qkv [T,Q] |
// pos [T] | LayerNorm row statistics [T][parts] (float2). The qkv region also
// holds the GeGLU output [T,I], so Q = max(3H, I) (I > 3H for a narrow model
// with a wide MLP, e.g. H 768 with I 2624).
int64_t qkv_cols(const lc_encoder_config& c) { return std::max<int64_t>(3 * (int64_t)c.hidden_size, c.intermediate_size); }
size_t pos_offset(const lc_encoder_config& c, int64_t T) { return (size_t)T * (2 * (size_t)c.hidden_size + (size_t)qkv_cols(c)) * 2; }
int stats_parts(const lc_encoder_config& c) {
  const int pc = gemm_stats_part_cols(c.hidden_size);
  return (c.hidden_size + pc - 1) / pc;
}
size_t stats_offset(const lc_encoder_config& c, int64_t T) {
  return (pos_offset(c, T) + (size_t)T * 4 + 255) & ~(size_t)255;
}
size_t workspace_bytes(const lc_encoder_config& c, int64_t T) {
  return stats_offset(c, T) + (size_t)T * stats_parts(c) * sizeof(float2);
}

// The forward on device ids (i32 [T]) and host cu_seqlens.
void forward(Encoder* e, const int32_t* ids_dev, const int32_t* cu, int nseq, LcTensor* hidden_out, const LcTensor* head_w,
             const LcTensor* head_b, float* probs_dev) {
  const lc_encoder_config& c = e->cfg;
  LC_CHECK(nseq > 0 && cu[0] == 0, "encoder: cu_seqlens must start at 0");
  int64_t T = cu[nseq];
  int maxlen = 0;
  for (int s = 0; s < nseq; s++) {
    LC_CHECK(cu[s + 1] >= cu[s], "encoder: cu_seqlens must be non-decreasing");
    maxlen = std::max(maxlen, cu[s + 1] - cu[s]);
  }
  LC_CHECK(T > 0, "encoder: empty batch");
  LC_CHECK(maxlen <= 8192, "encoder: sequences longer than 8192 tokens are not supported");
  const int H = c.hidden_size, I = c.intermediate_size;
  const int64_t esz = 2;
  cudaStream_t st = stream();
  // host-built metadata: cu_seqlens + attention tiles, one pinned staging buffer
  std::vector<int4> tiles = attention_tiles_tc(cu, nseq);
  size_t cu_bytes = ((size_t)(nseq + 1) * 4 + 15) & ~(size_t)15;
  size_t meta = cu_bytes + tiles.size() * sizeof(int4);
  if (e->stage_ev) CUDA_OK(cudaEventSynchronize(e->stage_ev));
  grow_pinned(e->stage, e->stage_bytes, meta);
  memcpy(e->stage, cu, (size_t)(nseq + 1) * 4);
  memcpy((char*)e->stage + cu_bytes, tiles.data(), tiles.size() * sizeof(int4));
  // workspace: the forward's buffers, then the metadata
  size_t off_meta = (workspace_bytes(c, T) + 255) & ~(size_t)255;
  grow_ws(e, off_meta + meta);
  char* ws = (char*)e->ws;
  int32_t* cu_dev = (int32_t*)(ws + off_meta);
  int4* tiles_dev = (int4*)(ws + off_meta + cu_bytes);
  CUDA_OK(cudaMemcpyAsync(ws + off_meta, e->stage, meta, cudaMemcpyHostToDevice, st));
  if (!e->stage_ev) CUDA_OK(cudaEventCreateWithFlags(&e->stage_ev, cudaEventDisableTiming));
  CUDA_OK(cudaEventRecord(e->stage_ev, st));
  (void)H, (void)I, (void)esz;
  run_kernels(e, ws, T, nseq, maxlen, cu_dev, tiles_dev, (int)tiles.size(), ids_dev, hidden_out ? hidden_out->data() : nullptr, head_w,
              head_b, probs_dev, st);
}

// The kernel sequence of one forward on prepared buffers: ws = x [T,H] | h [T,H] |
// qkv [T,max(3H,I)] | pos [T] | row statistics; cu_dev / tiles_dev on the device. Enqueues work only
// (no host synchronisation, no allocation once the encoder is warm), so a
// stream capture of it replays the forward.
void run_kernels(Encoder* e, char* ws, int64_t T, int nseq, int maxlen, const int32_t* cu_dev, const int4* tiles_dev, int ntiles,
                 const int32_t* ids_dev, void* hidden_out, const LcTensor* head_w, const LcTensor* head_b, float* probs_dev,
                 cudaStream_t st) {
  const lc_encoder_config& c = e->cfg;
  const int H = c.hidden_size, I = c.intermediate_size;
  const size_t esz = 2;
  void* x = ws;
  void* h = ws + (size_t)T * H * esz;
  void* qkv = ws + (size_t)2 * T * H * esz;
  int32_t* pos = (int32_t*)(ws + pos_offset(c, T));
  float2* stats = (float2*)(ws + stats_offset(c, T));
  const int parts = stats_parts(c), part_cols = gemm_stats_part_cols(H);
  // every kernel below waits for its predecessor on the device (pdl_wait)
  // and may be launched while that one still runs
  PdlScope pdl;
  launch_chain(k_positions, dim3(std::min(nseq, 4096)), dim3(256), 0, st, cu_dev, nseq, pos);
  LC_LAUNCHED(1);

  int cap_g = 0, cap_l = 0;
  const float* rope_g = rope_table(64, c.rope_theta_global, std::max(maxlen, 1), &cap_g, true);
  const float* rope_l = rope_table(64, c.rope_theta_local, std::max(maxlen, 1), &cap_l, true);

  // embeddings
  Prof* pe = new Prof(e, 2);
  unsigned lnb = blocks_for(T * 32, 256);
  const int per = (H / 8 + 31) / 32;
#define LC_EMB(TT, MV)                                                                                                    \
  launch_chain(k_embed_ln<TT, MV>, dim3(lnb), dim3(256), 0, st, (const TT*)e->tok->data(), e->tok->shape[0], ids_dev,        \
               (const float*)e->emb_norm->data(), (TT*)x, T, H, (float)c.norm_eps)
  if (c.dtype == LC_F16) {
    if (per <= 1) LC_EMB(__half, 1); else if (per <= 2) LC_EMB(__half, 2); else if (per <= 3) LC_EMB(__half, 3);
    else if (per <= 4) LC_EMB(__half, 4); else LC_EMB(__half, 8);
  } else {
    if (per <= 1) LC_EMB(__nv_bfloat16, 1); else if (per <= 2) LC_EMB(__nv_bfloat16, 2); else if (per <= 3) LC_EMB(__nv_bfloat16, 3);
    else if (per <= 4) LC_EMB(__nv_bfloat16, 4); else LC_EMB(__nv_bfloat16, 8);
  }
#undef LC_EMB
  LC_LAUNCHED(1);
  delete pe;

  const float scale = 1.0f / sqrtf(64.0f);
  // LayerNorms folded into the projection after them: the residual GEMMs
  // (Wo, mlp.Wo) record row statistics, the next projection normalises.
  auto folded = [&](GemmEpilogue& ep, const Mat& m) {
    ep.ln_stats = stats;
    ep.ln_wsum = (const float*)m.wsum->data();
    ep.ln_parts = parts;
    ep.ln_part_cols = part_cols;
    ep.ln_cols = H;
    ep.ln_eps = (float)c.norm_eps;
  };
  // Few rows: each GEMM brings the next projection's weight into L2 (the
  // chain is latency-bound there and the weights of all layers exceed L2).
  const bool l2_chain = T <= 4096;
  auto next_weight = [&](GemmEpilogue& ep, const Mat* m) {
    if (!l2_chain || !m) return;
    const LcTensor* t = m->dense ? m->dense : m->q;
    ep.l2_next = t->data();
    ep.l2_next_bytes = (size_t)t->numel() * dtype_size(t->dtype);
  };
  for (size_t li = 0; li < e->layers.size(); li++) {
    const Layer& L = e->layers[li];
    const Layer* Ln = li + 1 < e->layers.size() ? &e->layers[li + 1] : nullptr;
    const void* hin = x;
    GemmEpilogue eq;
    eq.kind = EPI_ROPE_QKV;
    eq.pos = pos;
    eq.rope_cs = L.kind == 0 ? rope_g : rope_l;
    eq.rope_cap = L.kind == 0 ? cap_g : cap_l;
    eq.rope_cols = 2 * H;
    if (L.attn_norm && L.Wqkv.wsum) {
      folded(eq, L.Wqkv);
    } else if (L.attn_norm) {  // a norm before the first layer: the embedding output has no statistics
      Prof p(e, 2);
      layernorm_raw(x, (const float*)L.attn_norm->data(), h, T, H, (float)c.norm_eps, c.dtype, st);
      hin = h;
    }
    next_weight(eq, &L.Wo);
    run_gemm(e, L.Wqkv, hin, T, qkv, 3 * H, eq, 3 * H, 0);
    // attention -> h (h is free again once the Wqkv GEMM has read it)
    {
      Prof p(e, 1);
      attention_varlen_tc(qkv, h, tiles_dev, ntiles, T, H, L.kind == 0 ? -1 : c.local_attention / 2, scale, c.dtype, st);
    }
    GemmEpilogue er;
    er.kind = EPI_RESIDUAL;
    er.resid = x;
    er.ldr = H;
    er.stats_out = stats;
    GemmEpilogue ero = er;
    next_weight(ero, &L.Wi);
    run_gemm(e, L.Wo, h, T, x, H, ero, H, 4);
    GemmEpilogue eg;
    eg.kind = EPI_GEGLU;
    folded(eg, L.Wi);
    next_weight(eg, &L.WoMlp);
    run_gemm(e, L.Wi, x, T, qkv, I, eg, I, 5);
    next_weight(er, Ln ? &Ln->Wqkv : nullptr);
    run_gemm(e, L.WoMlp, qkv, T, x, H, er, H, 6);
  }
  void* fin = hidden_out ? hidden_out : h;
  {
    Prof pf(e, 2);
    layernorm_raw(x, (const float*)e->final_norm->data(), fin, T, H, (float)c.norm_eps, c.dtype, st);
  }
  if (head_w && probs_dev) {
    Prof ph(e, 3);
    int C = (int)head_w->shape[0];
    size_t smem = C * sizeof(float);
    unsigned blocks = (unsigned)std::min(nseq, 65535);
    const char* hb = head_b ? (const char*)head_b->data() : nullptr;
    const int hbt = head_b ? head_b->dtype : 0;
    if (c.dtype == LC_F16)
      launch_chain(k_cls_head<__half>, dim3(blocks), dim3(128), smem, st, (const __half*)fin, H, cu_dev, nseq, (const char*)head_w->data(),
                   head_w->dtype, hb, hbt, C, probs_dev);
    else
      launch_chain(k_cls_head<__nv_bfloat16>, dim3(blocks), dim3(128), smem, st, (const __nv_bfloat16*)fin, H, cu_dev, nseq,
                   (const char*)head_w->data(), head_w->dtype, hb, hbt, C, probs_dev);
    LC_LAUNCHED(1);
  }
}

void check_head(const Encoder* e, const LcTensor* w, const LcTensor* b) {
  LC_CHECK(w->ndim == 2 && w->shape[1] == e->cfg.hidden_size && w->contiguous() && is_float(w->dtype) && w->dtype != LC_F64,
           "encoder: head_w must be a dense float [C, H] matrix");
  LC_CHECK(w->shape[0] >= 1 && w->shape[0] <= 4096, "encoder: 1..4096 classes");
  if (b) LC_CHECK(b->numel() == w->shape[0] && b->contiguous() && is_float(b->dtype) && b->dtype != LC_F64, "encoder: head_b must be [C]");
}

}  // namespace

extern "C" {

int lc_encoder_create(uint64_t* out, const lc_encoder_config* cfg, const int32_t* kinds, const lc_tensor* w, int nweights) {
  LC_API_BEGIN
  const lc_encoder_config& c = *cfg;
  LC_CHECK(c.dtype == LC_F16 || c.dtype == LC_BF16, "encoder: dtype must be f16 or bf16");
  LC_CHECK(c.num_heads > 0 && c.hidden_size == 64 * c.num_heads, "encoder: the fused path needs head dim 64");
  LC_CHECK(c.hidden_size % 64 == 0 && c.hidden_size <= 2048, "encoder: hidden size must be a multiple of 64, at most 2048");
  LC_CHECK(c.intermediate_size % 32 == 0 && c.intermediate_size % 8 == 0, "encoder: intermediate size must be a multiple of 32");
  LC_CHECK(c.num_layers >= 1 && c.vocab_size >= 1, "encoder: bad layer count / vocab");
  LC_CHECK(c.quant_bits == 0 || c.quant_bits == 4 || c.quant_bits == 8, "encoder: quant_bits must be 0, 4 or 8");
  int per = c.quant_bits ? 3 : 1;
  int want = 2 + c.num_layers * (2 + 4 * per) + 1;
  LC_CHECK(nweights == want, "encoder: expected " + std::to_string(want) + " weight handles, got " + std::to_string(nweights));
  auto e = std::make_unique<Encoder>();
  e->cfg = c;
  const int64_t H = c.hidden_size, I = c.intermediate_size, V = c.vocab_size;
  int i = 0;
  try {
    LcTensor* tok = check(w[i++], "encoder tok_embeddings");
    need_shape(tok, {V, H}, "tok_embeddings");
    LC_CHECK(tok->dtype == c.dtype, "encoder: tok_embeddings must be stored in the encoder dtype");
    e->tok = keep(e.get(), tok);
    LcTensor* en = check(w[i++], "encoder embeddings.norm");
    need_shape(en, {H}, "embeddings.norm");
    e->emb_norm = keep_f32(e.get(), en);
    for (int l = 0; l < c.num_layers; l++) {
      Layer L;
      L.kind = kinds[l];
      LC_CHECK(L.kind == 0 || L.kind == 1, "encoder: layer kind must be 0 (full) or 1 (sliding)");
      std::string p = "layers." + std::to_string(l) + ".";
      if (w[i]) {
        LcTensor* an = check(w[i], "encoder attn_norm");
        need_shape(an, {H}, p + "attn_norm");
        L.attn_norm = keep_f32(e.get(), an);
      } else {
        LC_CHECK(l == 0, "encoder: only layer 0 may omit attn_norm");
      }
      i++;
      L.Wqkv = take_mat(e.get(), w, i, 3 * H, H, p + "attn.Wqkv", false);
      L.Wo = take_mat(e.get(), w, i, H, H, p + "attn.Wo", false);
      LcTensor* mn = check(w[i++], "encoder mlp_norm");
      need_shape(mn, {H}, p + "mlp_norm");
      L.mlp_norm = keep_f32(e.get(), mn);
      L.Wi = take_mat(e.get(), w, i, 2 * I, H, p + "mlp.Wi", true);
      L.WoMlp = take_mat(e.get(), w, i, H, I, p + "mlp.Wo", false);
      if (l > 0) fold_norm(e.get(), L.Wqkv, L.attn_norm);
      fold_norm(e.get(), L.Wi, L.mlp_norm);
      e->layers.push_back(L);
    }
    LcTensor* fn = check(w[i++], "encoder final_norm");
    need_shape(fn, {H}, "final_norm");
    e->final_norm = keep_f32(e.get(), fn);
    // RoPE tables for every position the model can see (no growth during a forward)
    int cap;
    rope_table(64, c.rope_theta_global, 8192, &cap, true);
    rope_table(64, c.rope_theta_local, 8192, &cap, true);
  } catch (...) {
    for (auto* t : e->owned) release(t);
    throw;
  }
  Encoder* raw = e.release();
  encoders().insert(raw);
  *out = reinterpret_cast<uint64_t>(raw);
  LC_API_END
}

int lc_encoder_free(uint64_t h) {
  LC_API_BEGIN
  Encoder* e = check_enc(h);
  encoders().erase(e);
  CUDA_OK(cudaStreamSynchronize(stream()));
  free_graphs_of(e);
  for (auto* t : e->owned) release(t);
  if (e->deq) release(e->deq);
  if (e->ws) dfree(e->ws);
  if (e->stage) cudaFreeHost(e->stage);
  if (e->ids_stage) cudaFreeHost(e->ids_stage);
  if (e->probs_stage) cudaFreeHost(e->probs_stage);
  if (e->stage_ev) cudaEventDestroy(e->stage_ev);
  for (auto& pe : e->pending) cudaEventDestroy(pe.second.first), cudaEventDestroy(pe.second.second);
  for (auto ev : e->ev_pool) cudaEventDestroy(ev);
  delete e;
  LC_API_END
}

int lc_encoder_set_profiling(uint64_t h, int on) {
  LC_API_BEGIN
  check_enc(h)->prof = on != 0;
  LC_API_END
}

int lc_encoder_profile_read(uint64_t h, double* ms, int64_t* n) {
  LC_API_BEGIN
  Encoder* e = check_enc(h);
  CUDA_OK(cudaStreamSynchronize(stream()));
  for (auto& pe : e->pending) {
    float t = 0.f;
    CUDA_OK(cudaEventElapsedTime(&t, pe.second.first, pe.second.second));
    e->prof_ms[pe.first] += t;
    e->prof_n[pe.first] += 1;
    e->ev_pool.push_back(pe.second.first);
    e->ev_pool.push_back(pe.second.second);
  }
  e->pending.clear();
  for (int i = 0; i < 8; i++) {
    ms[i] = e->prof_ms[i];
    n[i] = e->prof_n[i];
    e->prof_ms[i] = 0;
    e->prof_n[i] = 0;
  }
  LC_API_END
}

int lc_encoder_forward(lc_tensor* hidden, lc_tensor* probs, uint64_t h, lc_tensor idsh, const int32_t* cu, int nseq, lc_tensor hwh,
                       lc_tensor hbh) {
  LC_API_BEGIN
  Encoder* e = check_enc(h);
  LcTensor* ids = check(idsh, "encoder ids");
  LC_CHECK(ids->dtype == LC_I32 && ids->contiguous() && ids->numel() == cu[nseq], "encoder: ids must be dense i32 [T] with T = cu_seqlens[nseq]");
  LcTensor* hw = hwh ? check(hwh, "encoder head_w") : nullptr;
  LcTensor* hb = hbh ? check(hbh, "encoder head_b") : nullptr;
  if (hw) check_head(e, hw, hb);
  LC_CHECK(!probs || hw, "encoder: probs need head_w");
  LcTensor* hid = hidden ? alloc(e->cfg.dtype, {(int64_t)cu[nseq], (int64_t)e->cfg.hidden_size}) : nullptr;
  LcTensor* pr = probs ? alloc(LC_F32, {(int64_t)nseq, hw->shape[0]}) : nullptr;
  try {
    forward(e, (const int32_t*)ids->data(), cu, nseq, hid, hw, hb, pr ? (float*)pr->data() : nullptr);
  } catch (...) {
    if (hid) release(hid);
    if (pr) release(pr);
    throw;
  }
  if (hidden) *hidden = handle(hid);
  if (probs) *probs = handle(pr);
  LC_API_END
}

int lc_encoder_forward_host(uint64_t h, const int32_t* ids_host, const int32_t* cu, int nseq, lc_tensor hwh, lc_tensor hbh, float* probs_host) {
  LC_API_BEGIN
  Encoder* e = check_enc(h);
  LcTensor* hw = check(hwh, "encoder head_w");
  LcTensor* hb = hbh ? check(hbh, "encoder head_b") : nullptr;
  check_head(e, hw, hb);
  LC_CHECK(nseq > 0 && cu[0] == 0, "encoder: cu_seqlens must start at 0");
  int64_t T = cu[nseq];
  int64_t C = hw->shape[0];
  cudaStream_t st = stream();
  // ids: host -> pinned staging -> device
  grow_pinned(e->ids_stage, e->ids_stage_bytes, (size_t)T * 4);
  if (e->stage_ev) CUDA_OK(cudaEventSynchronize(e->stage_ev));
  memcpy(e->ids_stage, ids_host, (size_t)T * 4);
  int32_t* ids_dev = (int32_t*)dmalloc((size_t)T * 4);
  float* probs_dev = (float*)dmalloc((size_t)nseq * C * 4);
  CUDA_OK(cudaMemcpyAsync(ids_dev, e->ids_stage, (size_t)T * 4, cudaMemcpyHostToDevice, st));
  try {
    forward(e, ids_dev, cu, nseq, nullptr, hw, hb, probs_dev);
  } catch (...) {
    dfree(ids_dev);
    dfree(probs_dev);
    throw;
  }
  grow_pinned(e->probs_stage, e->probs_stage_bytes, (size_t)nseq * C * 4);
  CUDA_OK(cudaMemcpyAsync(e->probs_stage, probs_dev, (size_t)nseq * C * 4, cudaMemcpyDeviceToHost, st));
  dfree(ids_dev);
  dfree(probs_dev);
  CUDA_OK(cudaStreamSynchronize(st));
  memcpy(probs_host, e->probs_stage, (size_t)nseq * C * 4);
  std::string err = take_device_errors();
  LC_CHECK(err.empty(), err);
  LC_API_END
}

}  // extern "C"

// ------------------------------------------------------------- CUDA-graph replay
// One fixed batch shape (cu_seqlens) captured as a graph: H2D of the ids from
// the graph's pinned buffer, the whole forward, D2H of the probabilities. The
// graph owns its workspace, metadata and I/O buffers, so eager forwards of the
// same encoder can run in between.

namespace {
struct EncGraph {
  Encoder* e = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  char* ws = nullptr;
  char* meta = nullptr;
  int32_t* ids_dev = nullptr;
  float* probs_dev = nullptr;
  void* ids_pin = nullptr;
  void* probs_pin = nullptr;
  int64_t T = 0;
  int nseq = 0, C = 0;
};
std::unordered_set<EncGraph*>& graphs() {
  static std::unordered_set<EncGraph*> s;
  return s;
}
void free_graph(EncGraph* g) {
  if (g->exec) cudaGraphExecDestroy(g->exec);
  if (g->graph) cudaGraphDestroy(g->graph);
  cudaStreamSynchronize(stream());
  for (void* p : {(void*)g->ws, (void*)g->meta, (void*)g->ids_dev, (void*)g->probs_dev}) dfree(p);
  if (g->ids_pin) cudaFreeHost(g->ids_pin);
  if (g->probs_pin) cudaFreeHost(g->probs_pin);
  delete g;
}

void free_graphs_of(Encoder* e) {
  for (auto it = graphs().begin(); it != graphs().end();) {
    if ((*it)->e == e) {
      free_graph(*it);
      it = graphs().erase(it);
    } else {
      ++it;
    }
  }
}
}  // namespace

extern "C" {

int lc_encoder_graph_create(uint64_t* out, uint64_t h, const int32_t* cu, int nseq, lc_tensor hwh, lc_tensor hbh) {
  LC_API_BEGIN
  Encoder* e = check_enc(h);
  LcTensor* hw = check(hwh, "encoder graph head_w");
  LcTensor* hb = hbh ? check(hbh, "encoder graph head_b") : nullptr;
  check_head(e, hw, hb);
  LC_CHECK(nseq > 0 && cu[0] == 0, "encoder graph: cu_seqlens must start at 0");
  int maxlen = 0;
  for (int s = 0; s < nseq; s++) {
    LC_CHECK(cu[s + 1] >= cu[s], "encoder graph: cu_seqlens must be non-decreasing");
    maxlen = std::max(maxlen, cu[s + 1] - cu[s]);
  }
  LC_CHECK(cu[nseq] > 0 && maxlen <= 8192, "encoder graph: 1..8192 tokens per sequence");
  auto g = std::make_unique<EncGraph>();
  g->e = e;
  g->T = cu[nseq];
  g->nseq = nseq;
  g->C = (int)hw->shape[0];
  cudaStream_t st = stream();
  std::vector<int4> tiles = attention_tiles_tc(cu, nseq);
  size_t cu_bytes = ((size_t)(nseq + 1) * 4 + 15) & ~(size_t)15;
  size_t meta = cu_bytes + tiles.size() * sizeof(int4);
  try {
    g->ws = (char*)dmalloc(workspace_bytes(e->cfg, g->T));
    g->meta = (char*)dmalloc(meta);
    g->ids_dev = (int32_t*)dmalloc((size_t)g->T * 4);
    g->probs_dev = (float*)dmalloc((size_t)nseq * g->C * 4);
    CUDA_OK(cudaHostAlloc(&g->ids_pin, (size_t)g->T * 4, cudaHostAllocDefault));
    CUDA_OK(cudaHostAlloc(&g->probs_pin, (size_t)nseq * g->C * 4, cudaHostAllocDefault));
    std::vector<char> hmeta(meta, 0);
    memcpy(hmeta.data(), cu, (size_t)(nseq + 1) * 4);
    memcpy(hmeta.data() + cu_bytes, tiles.data(), tiles.size() * sizeof(int4));
    CUDA_OK(cudaMemcpyAsync(g->meta, hmeta.data(), meta, cudaMemcpyHostToDevice, st));
    CUDA_OK(cudaMemsetAsync(g->ids_dev, 0, (size_t)g->T * 4, st));
    memset(g->ids_pin, 0, (size_t)g->T * 4);
    const int32_t* cu_dev = (const int32_t*)g->meta;
    const int4* tiles_dev = (const int4*)(g->meta + cu_bytes);
    // warm-up outside the capture: tensor maps, kernel attributes, dequant scratch
    const bool prof = e->prof;
    e->prof = false;
    run_kernels(e, g->ws, g->T, nseq, maxlen, cu_dev, tiles_dev, (int)tiles.size(), g->ids_dev, nullptr, hw, hb, g->probs_dev, st);
    CUDA_OK(cudaStreamSynchronize(st));
    CUDA_OK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    try {
      CUDA_OK(cudaMemcpyAsync(g->ids_dev, g->ids_pin, (size_t)g->T * 4, cudaMemcpyHostToDevice, st));
      run_kernels(e, g->ws, g->T, nseq, maxlen, cu_dev, tiles_dev, (int)tiles.size(), g->ids_dev, nullptr, hw, hb, g->probs_dev, st);
      CUDA_OK(cudaMemcpyAsync(g->probs_pin, g->probs_dev, (size_t)nseq * g->C * 4, cudaMemcpyDeviceToHost, st));
    } catch (...) {
      cudaGraph_t dead = nullptr;
      cudaStreamEndCapture(st, &dead);
      if (dead) cudaGraphDestroy(dead);
      e->prof = prof;
      throw;
    }
    CUDA_OK(cudaStreamEndCapture(st, &g->graph));
    e->prof = prof;
    CUDA_OK(cudaGraphInstantiate(&g->exec, g->graph, 0));
  } catch (...) {
    free_graph(g.release());
    throw;
  }
  EncGraph* raw = g.release();
  graphs().insert(raw);
  *out = reinterpret_cast<uint64_t>(raw);
  LC_API_END
}

int lc_encoder_graph_run(uint64_t gh, const int32_t* ids_host, float* probs_host) {
  LC_API_BEGIN
  EncGraph* g = reinterpret_cast<EncGraph*>(gh);
  LC_CHECK(gh && graphs().count(g), "encoder graph: invalid or freed graph handle");
  memcpy(g->ids_pin, ids_host, (size_t)g->T * 4);
  CUDA_OK(cudaGraphLaunch(g->exec, stream()));
  CUDA_OK(cudaStreamSynchronize(stream()));
  memcpy(probs_host, g->probs_pin, (size_t)g->nseq * g->C * 4);
  std::string err = take_device_errors();
  LC_CHECK(err.empty(), err);
  LC_API_END
}

int lc_encoder_graph_free(uint64_t gh) {
  LC_API_BEGIN
  EncGraph* g = reinterpret_cast<EncGraph*>(gh);
  LC_CHECK(gh && graphs().count(g), "encoder graph: invalid or freed graph handle");
  graphs().erase(g);
  free_graph(g);
  LC_API_END
}

}  // extern "C"

// Sets this unit's bounded-wait limit (lc_debug_set_wait_limit).
void lc_internal_wait_limit_encoder(unsigned long long ns) { CUDA_OK(cudaMemcpyToSymbol(sm100::g_wait_limit_ns, &ns, sizeof(ns))); }
