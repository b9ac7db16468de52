// Quantized weights: the optional trio fromHostQuantized / quantizedLinear /
// quantizedEmbedding (packages/tensor-backend/src/index.ts:247-263).
//
// Native layout = the laya-js checkpoint bytes as-is (index.ts:98-108): rows
// of K·bits/8 bytes, 4-bit values two per byte with the even column in the
// low nibble (read as little-endian u32 words this is MLX's packing). Scales
// and biases [N, ceil(K/g)] are stored in the dequantisation dtype.
//
// Every dequantised value is fl(q·s + b) rounded ONCE to the target dtype,
// the rule of the reference's host dequantiser (packages/laya/src/quant.ts:189-243),
// which computes q·s + b in JS doubles and stores the double into the typed
// array: here q·s + b is one f64 FMA (q·s is exact in f64, so the only
// rounding before the store is the FMA's own, as in the reference's double
// expression) and the double is then rounded once to f32, f16 or bf16
// (dequant_f64 / store_dequant in lc_quant.cuh).
#include "lc_api.h"
#include "lc_gemm.h"
#include "lc_quant.cuh"

#include <mutex>

using namespace lc;

// ------------------------------------------------------------- kernels

// dequantise rows [N, K] -> out [N, K] in out dtype
__global__ void k_dequant(const uint8_t* __restrict__ w, const char* s, const char* b, int sdt, int bits, int g, int mode, int64_t N,
                          int64_t K, char* out, int odt) {
  pdl_trigger();
  pdl_wait();
  int64_t G = (K + g - 1) / g;
  LC_GRID_STRIDE(t, N * K) {
    int64_t r = t / K, j = t % K;
    int q = quant_value(w + r * (K * bits / 8), j, bits, mode);
    float sv = ld_as<float>(s, sdt, r * G + j / g);
    float bv = b ? ld_as<float>(b, sdt, r * G + j / g) : 0.f;
    store_dequant(out, odt, t, q, sv, bv);
  }
}

// dequantise rows [N, K] into 16-bit `out` with column k scaled by gamma[k]:
// out = round(round(q·s + b) · γ_k) — the weight the encoder's folded
// LayerNorm multiplies by (the dense path folds the stored weight the same way)
__global__ void k_dequant_scaled(const uint8_t* __restrict__ w, const char* s, const char* b, int sdt, int bits, int g, int mode, int64_t N,
                                 int64_t K, const float* __restrict__ gamma, char* out, int odt) {
  pdl_trigger();
  pdl_wait();
  int64_t G = (K + g - 1) / g;
  LC_GRID_STRIDE(t, N * K) {
    int64_t r = t / K, j = t % K;
    int q = quant_value(w + r * (K * bits / 8), j, bits, mode);
    float sv = ld_as<float>(s, sdt, r * G + j / g);
    float bv = b ? ld_as<float>(b, sdt, r * G + j / g) : 0.f;
    st_as<float>(out, odt, t, dequant_rounded(odt, q, sv, bv) * gamma[j]);
  }
}

// row gather + dequantise: out [n, K], row i = dequant(w[ids[i]]) (zeros for an out-of-range id)
__global__ void k_quant_gather(const uint8_t* __restrict__ w, const char* s, const char* b, int sdt, int bits, int g, int mode, int64_t V,
                               int64_t K, const char* ids, int iddt, int64_t n, char* out, int odt) {
  int64_t G = (K + g - 1) / g;
  LC_GRID_STRIDE(t, n * K) {
    int64_t i = t / K, j = t % K;
    int64_t r = ld_as<int64_t>(ids, iddt, i);
    if (r < 0 || r >= V) {
      st_as<float>(out, odt, t, 0.f);
      continue;
    }
    int q = quant_value(w + r * (K * bits / 8), j, bits, mode);
    float sv = ld_as<float>(s, sdt, r * G + j / g);
    float bv = b ? ld_as<float>(b, sdt, r * G + j / g) : 0.f;
    store_dequant(out, odt, t, q, sv, bv);
  }
}

// Small-M quantized linear: one warp per output feature n, reading the packed
// row once for all M (<= 8) input rows; f32 accumulation. The dequantised
// weight is rounded to x's dtype first (it is the weight the contract's
// composition multiplies by: compose.ts:407-417).
template <int MMAX>
__global__ void k_qgemv(const char* x, int xdt, int64_t M, const uint8_t* __restrict__ w, const char* s, const char* b, int sdt, int bits,
                        int g, int mode, int64_t N, int64_t K, const char* bias, int biasdt, char* y, int ydt) {
  int lane = threadIdx.x & 31;
  int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  int64_t G = (K + g - 1) / g;
  for (int64_t n = warp; n < N; n += nwarps) {
    float acc[MMAX];
#pragma unroll
    for (int m = 0; m < MMAX; m++) acc[m] = 0.f;
    const uint8_t* row = w + n * (K * bits / 8);
    for (int64_t j = lane; j < K; j += 32) {
      int q = quant_value(row, j, bits, mode);
      float sv = ld_as<float>(s, sdt, n * G + j / g);
      float bv = b ? ld_as<float>(b, sdt, n * G + j / g) : 0.f;
      float wv = dequant_rounded(xdt, q, sv, bv);
#pragma unroll
      for (int m = 0; m < MMAX; m++)
        if (m < M) acc[m] += ld_as<float>(x, xdt, m * K + j) * wv;
    }
#pragma unroll
    for (int m = 0; m < MMAX; m++) {
      float v = acc[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0 && m < M) {
        if (bias) v += ld_as<float>(bias, biasdt, n);
        st_as<float>(y, ydt, m * N + n, v);
      }
    }
  }
}

namespace {

void validate(int64_t n, int64_t k, int bits, int g, int mode) {
  std::string where = "quantized [" + std::to_string(n) + ", " + std::to_string(k) + "] q" + std::to_string(bits) + "/g" + std::to_string(g);
  LC_CHECK(bits == 4 || bits == 8, where + ": bits must be 4 or 8");
  LC_CHECK(mode == 0 || mode == 1, where + ": mode must be symmetric (0) or affine (1)");
  LC_CHECK(n > 0 && k > 0, where + ": bad shape");
  LC_CHECK(g > 0, where + ": bad group size");
  LC_CHECK((k * bits) % 32 == 0, where + ": in · bits must be a multiple of 32");
}

struct QW {
  LcTensor *w, *s, *b;
  int64_t N, K, G;
};

QW check_q(uint64_t wh, uint64_t sh, uint64_t bh, int bits, int g, int mode, const char* name) {
  QW q;
  q.w = check(wh, name);
  q.s = check(sh, name);
  q.b = bh ? check(bh, name) : nullptr;
  LC_CHECK(q.w->dtype == LC_U8 && q.w->ndim == 2 && q.w->contiguous(), std::string(name) + ": weight is not a native packed matrix");
  q.N = q.w->shape[0];
  q.K = q.w->shape[1] * 8 / bits;
  validate(q.N, q.K, bits, g, mode);
  q.G = (q.K + g - 1) / g;
  LC_CHECK(q.s->ndim == 2 && q.s->shape[0] == q.N && q.s->shape[1] == q.G && q.s->contiguous(), std::string(name) + ": scales shape");
  if (mode == 1) LC_CHECK(q.b && q.b->ndim == 2 && q.b->shape[0] == q.N && q.b->shape[1] == q.G && q.b->contiguous(), std::string(name) + ": biases");
  else LC_CHECK(!q.b, std::string(name) + ": symmetric quantization takes no biases");
  return q;
}

}  // namespace

namespace lc {
// Dequantise the whole matrix into `out` [N, K] (dense, dtype = out->dtype).
void dequant_into(const LcTensor* w, const LcTensor* s, const LcTensor* b, int bits, int g, int mode, LcTensor* out) {
  int64_t N = w->shape[0], K = w->shape[1] * 8 / bits;
  launch_chain(k_dequant, dim3(blocks_for(N * K, 256)), dim3(256), 0, stream(), (const uint8_t*)w->data(), (const char*)s->data(),
               b ? (const char*)b->data() : nullptr, s->dtype, bits, g, mode, N, K, (char*)out->data(), out->dtype);
  LC_LAUNCHED(1);
}
// The same with column k scaled by gamma[k] (f32, K values), out f16/bf16.
void dequant_scaled_into(const LcTensor* w, const LcTensor* s, const LcTensor* b, int bits, int g, int mode, const float* gamma, LcTensor* out) {
  int64_t N = w->shape[0], K = w->shape[1] * 8 / bits;
  launch_chain(k_dequant_scaled, dim3(blocks_for(N * K, 256)), dim3(256), 0, stream(), (const uint8_t*)w->data(), (const char*)s->data(),
               b ? (const char*)b->data() : nullptr, s->dtype, bits, g, mode, N, K, gamma, (char*)out->data(), out->dtype);
  LC_LAUNCHED(1);
}
}  // namespace lc

extern "C" {

int lc_from_host_quantized(lc_tensor* wout, lc_tensor* sout, lc_tensor* bout, int64_t n, int64_t k, int bits, int group_size, int mode,
                           const uint8_t* data, int sb_dtype, const void* scales_host, const void* biases_host, int dtype) {
  LC_API_BEGIN
  validate(n, k, bits, group_size, mode);
  LC_CHECK(is_float(dtype) && dtype != LC_F64, "fromHostQuantized: dtype must be f32, f16 or bf16");
  LC_CHECK(sb_dtype == LC_F32 || sb_dtype == LC_F16 || sb_dtype == LC_BF16, "fromHostQuantized: scales must be float");
  LC_CHECK(mode == 1 ? biases_host != nullptr : biases_host == nullptr,
           mode == 1 ? "fromHostQuantized: affine quantization needs biases" : "fromHostQuantized: symmetric quantization takes no biases");
  int64_t G = (k + group_size - 1) / group_size;
  int64_t rowbytes = k * bits / 8;
  lc_tensor w = 0, s0 = 0, b0 = 0, s = 0, b = 0;
  int64_t wsh[2] = {n, rowbytes}, ssh[2] = {n, G};
  if (lc_from_host(&w, LC_U8, wsh, 2, data, (size_t)(n * rowbytes))) throw Error(lc_last_error());
  if (lc_from_host(&s0, sb_dtype, ssh, 2, scales_host, (size_t)(n * G * dtype_size(sb_dtype)))) throw Error(lc_last_error());
  if (sb_dtype != dtype) {
    if (lc_cast(&s, s0, dtype)) throw Error(lc_last_error());
    lc_tensor_free(s0);
  } else s = s0;
  if (mode == 1) {
    if (lc_from_host(&b0, sb_dtype, ssh, 2, biases_host, (size_t)(n * G * dtype_size(sb_dtype)))) throw Error(lc_last_error());
    if (sb_dtype != dtype) {
      if (lc_cast(&b, b0, dtype)) throw Error(lc_last_error());
      lc_tensor_free(b0);
    } else b = b0;
  }
  *wout = w;
  *sout = s;
  *bout = b;
  LC_API_END
}

int lc_dequantize(lc_tensor* out, lc_tensor wh, lc_tensor sh, lc_tensor bh, int bits, int g, int mode) {
  LC_API_BEGIN
  QW q = check_q(wh, sh, bh, bits, g, mode, "dequantize");
  LcTensor* y = alloc(q.s->dtype, {q.N, q.K});
  dequant_into(q.w, q.s, q.b, bits, g, mode, y);
  *out = handle(y);
  LC_API_END
}

int lc_quantized_embedding(lc_tensor* out, lc_tensor wh, lc_tensor sh, lc_tensor bh, int bits, int g, int mode, lc_tensor ih) {
  LC_API_BEGIN
  QW q = check_q(wh, sh, bh, bits, g, mode, "quantizedEmbedding");
  LcTensor* ids0 = check(ih, "quantizedEmbedding ids");
  LC_CHECK(!is_float(ids0->dtype), "quantizedEmbedding: ids must be integers");
  std::vector<int64_t> osh = ids0->dims();
  osh.push_back(q.K);
  LcTensor* y = alloc(q.s->dtype, osh);
  int64_t n = ids0->numel();
  if (n) {
    LcTensor* ids = contiguous(ids0);
    k_quant_gather<<<blocks_for(n * q.K, 256), 256, 0, stream()>>>((const uint8_t*)q.w->data(), q.s->data(), q.b ? q.b->data() : nullptr,
                                                                  q.s->dtype, bits, g, mode, q.N, q.K, ids->data(), ids->dtype, n, y->data(),
                                                                  y->dtype);
    LC_LAUNCHED(1);
    if (ids != ids0) release(ids);
  }
  *out = handle(y);
  LC_API_END
}

// y = x · dequant(w)ᵀ (+ bias) with the dequantisation inside the GEMM, when
// the shape suits it (few rows); false when nothing was launched.
static bool fused_q(const LcTensor* x, const QW& q, int bits, int g, int mode, const LcTensor* bias, LcTensor* y, int64_t M) {
  GemmQuantB qb;
  qb.w = (const uint8_t*)q.w->data();
  qb.scales = q.s->data();
  qb.biases = q.b ? q.b->data() : nullptr;
  qb.sdt = q.s->dtype;
  qb.bits = bits;
  qb.group = g;
  qb.mode = mode;
  return gemm_raw_q(x->data(), M, q.K, qb, q.N, bias ? bias->data() : nullptr, bias ? bias->dtype : 0, y->data(), q.N, y->dtype,
                    GemmEpilogue{}, stream());
}

int lc_quantized_linear(lc_tensor* out, lc_tensor xh, lc_tensor wh, lc_tensor sh, lc_tensor bh, int bits, int g, int mode, lc_tensor biash) {
  LC_API_BEGIN
  QW q = check_q(wh, sh, bh, bits, g, mode, "quantizedLinear");
  LcTensor* x0 = check(xh, "quantizedLinear x");
  LcTensor* bias0 = biash ? check(biash, "quantizedLinear bias") : nullptr;
  LC_CHECK(x0->ndim >= 1 && x0->shape[x0->ndim - 1] == q.K, "quantizedLinear: x [" + shape_str(x0->dims()) + "] vs w [" + std::to_string(q.N) + ", " + std::to_string(q.K) + "]");
  if (bias0) LC_CHECK(bias0->numel() == q.N, "quantizedLinear: bias size differs from out features");
  int odt = is_float(x0->dtype) ? x0->dtype : LC_F32;
  std::vector<int64_t> osh = x0->dims();
  osh.back() = q.N;
  LcTensor* y = alloc(odt, osh);
  int64_t M = x0->numel() / q.K;
  if (M) {
    LcTensor* x = contiguous(x0);
    LcTensor* bias = bias0 ? contiguous(bias0) : nullptr;
    if (M <= 8) {
      unsigned blocks = blocks_for(q.N * 32, 256);
      k_qgemv<8><<<blocks, 256, 0, stream()>>>(x->data(), x->dtype, M, (const uint8_t*)q.w->data(), q.s->data(), q.b ? q.b->data() : nullptr,
                                                q.s->dtype, bits, g, mode, q.N, q.K, bias ? bias->data() : nullptr, bias ? bias->dtype : 0,
                                                y->data(), odt);
      LC_LAUNCHED(1);
    } else if (is_half(odt) && x->dtype == odt && fused_q(x, q, bits, g, mode, bias, y, M)) {
      // few rows: dequantised inside the tcgen05 GEMM
    } else {
      // dequantise once into x's dtype (scratch), then the dense GEMM
      LcTensor* wd = alloc(odt, {q.N, q.K});
      dequant_into(q.w, q.s, q.b, bits, g, mode, wd);
      LcTensor* x2 = view_of(x, {M, q.K}, {q.K, 1}, x->offset);
      bool done = false;
      if (is_half(odt) && x->dtype == odt) done = gemm_linear(x2, wd, bias, y, GemmEpilogue{});
      if (!done) {
        LcTensor* y2 = view_of(y, {M, q.N}, {q.N, 1}, 0);
        linear_simt(x2, wd, bias, y2);
        release(y2);
      }
      release(x2);
      release(wd);
    }
    if (x != x0) release(x);
    if (bias && bias != bias0) release(bias);
  }
  *out = handle(y);
  LC_API_END
}

}  // extern "C"

// ------------------------------------------------------------- allocation-free quantized linear
//
// lc_quantized_linear_noalloc is for callers that cannot allocate device memory
// themselves: for example a host whose device memory is all handed to another
// framework's caching allocator, or a serving loop that must not call
// cudaMalloc / cudaFree (they can synchronise the whole device) on its hot
// path. It computes the same y = x · dequant(w)ᵀ (+ bias) as
// lc_quantized_linear's large-M path (dequantise once, then the tcgen05 GEMM),
// but the dequantised weight goes into the fixed scratch array below instead of
// an allocation; the caller passes device pointers for every input and output.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes: every
// GPU that loads this library reserves it until the process exits. Host code
// cannot use the array's name as a device address, so the first call on each
// device looks the address up with cudaGetSymbolAddress (with that device
// current) and keeps it; make that first call before any stream capture. All
// calls share the one array and it keeps the last call's contents: each call
// overwrites exactly the N·K values it reads, so nothing needs clearing, but
// calls that overlap on the GPU (different streams, no ordering between them)
// race on it. Like every other entry of this library, calls are expected from
// one host thread at a time (the GEMM's tensor-map cache is not locked).

static constexpr size_t kNoAllocScratchBytes = (size_t)8 << 20;  // room for a 4M-element f16/bf16 weight
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
// The scratch address of the current device, looked up once per device. The
// mutex keeps two host threads that make their first call at the same time
// from racing on the table.
void* noalloc_scratch_for_current_device() {
  static void* ptrs[128] = {};
  static std::mutex mu;
  int dev = -1;
  CUDA_OK(cudaGetDevice(&dev));
  LC_CHECK(dev >= 0 && dev < 128, "quantizedLinearNoalloc: device ordinal out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    CUDA_OK(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    LC_CHECK(p != nullptr, "quantizedLinearNoalloc: cudaGetSymbolAddress returned no address for the scratch array");
    ptrs[dev] = p;
  }
  return ptrs[dev];
}
}  // namespace

extern "C" int lc_quantized_linear_noalloc(void* y, const void* x, int64_t m, int64_t k, int dtype, const uint8_t* w, const void* scales,
                                           const void* biases, int64_t n, int bits, int group_size, int mode, int sb_dtype,
                                           const void* bias, int bias_dtype, uint64_t stream) {
  LC_API_BEGIN
  validate(n, k, bits, group_size, mode);
  LC_CHECK(dtype == LC_F16 || dtype == LC_BF16, "quantizedLinearNoalloc: x and y must be f16 or bf16");
  LC_CHECK(sb_dtype == LC_F32 || sb_dtype == LC_F16 || sb_dtype == LC_BF16, "quantizedLinearNoalloc: scales/biases must be f32, f16 or bf16");
  LC_CHECK(mode == 1 ? biases != nullptr : biases == nullptr, "quantizedLinearNoalloc: biases are required for affine and not allowed for symmetric");
  LC_CHECK(!bias || bias_dtype == LC_F32 || bias_dtype == LC_F16 || bias_dtype == LC_BF16,
           "quantizedLinearNoalloc: bias must be f32, f16 or bf16");
  LC_CHECK(x && y && w && scales && m > 0, "quantizedLinearNoalloc: null pointer or empty input");
  LC_CHECK(k >= 64 && k % 8 == 0, "quantizedLinearNoalloc: in features must be a multiple of 8, at least 64");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // few rows: dequantised inside the GEMM, no scratch
  GemmQuantB qb;
  qb.w = w;
  qb.scales = scales;
  qb.biases = biases;
  qb.sdt = sb_dtype;
  qb.bits = bits;
  qb.group = group_size;
  qb.mode = mode;
  if (gemm_raw_q(x, m, k, qb, n, bias, bias_dtype, y, n, dtype, GemmEpilogue{}, st)) return 0;
  const size_t need = (size_t)n * (size_t)k * 2;
  LC_CHECK(need <= kNoAllocScratchBytes,
           "quantizedLinearNoalloc: the dequantised weight needs " + std::to_string(need) + " bytes, above the " +
               std::to_string(kNoAllocScratchBytes) + "-byte scratch (out x in <= " + std::to_string(kNoAllocScratchBytes / 2) + ")");
  void* scratch = noalloc_scratch_for_current_device();
  k_dequant<<<blocks_for(n * k, 256), 256, 0, st>>>(w, (const char*)scales, (const char*)biases, sb_dtype, bits, group_size, mode, n, k,
                                                    (char*)scratch, dtype);
  LC_LAUNCHED(1);
  bool ok = gemm_raw(x, m, k, scratch, n, bias, bias_dtype, y, n, dtype, GemmEpilogue{}, st);
  LC_CHECK(ok, "quantizedLinearNoalloc: shape or alignment not supported by the tensor-core GEMM (16-byte aligned pointers needed)");
  LC_API_END
}
