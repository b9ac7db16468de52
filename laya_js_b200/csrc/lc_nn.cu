// NN ops of the contract that are not the tensor-core GEMM:
// layerNorm, embedding, gatherRows, rope, sdpa (generic), geglu, meanPool,
// matmul and the exact-f32 SIMT linear used for f32/f64 and shapes the
// tcgen05 GEMM does not take (packages/tensor-backend/src/index.ts:208-243).
#include "lc_api.h"
#include "lc_gelu.cuh"
#include "lc_gemm.h"

#include <cmath>
#include <map>
#include <tuple>

using namespace lc;

// ------------------------------------------------------------- layerNorm
// index.ts:216-217: normalise over the last axis, stats in f32, optional weight/bias.

// Four LayerNorm weights (or biases) as floats: f32, or the rows' own 16-bit type.
template <typename WT>
__device__ __forceinline__ float4 ld_w4(const WT* p, int64_t i, float fill) {
  if (!p) return make_float4(fill, fill, fill, fill);
  if constexpr (sizeof(WT) == 4) {
    return __ldg((const float4*)(p + i));
  } else {
    const uint2 u = __ldg((const uint2*)(p + i));
    const WT* h = (const WT*)&u;
    return make_float4(to_f<WT>(h[0]), to_f<WT>(h[1]), to_f<WT>(h[2]), to_f<WT>(h[3]));
  }
}

// Vectorised fast path: dense f16/bf16/f32 rows, N % 8 == 0 (f32: % 4), N <= 256 vectors;
// weight and bias f32 or of the rows' type (WT). A warp takes R rows at a time
// (R = 2 for short rows: both rows' loads in flight together, their
// reductions interleaved).
template <typename T, int MAXV, typename WT = float>
__global__ void __launch_bounds__(256) k_layernorm_vec(const T* __restrict__ x, const WT* __restrict__ w, const WT* __restrict__ b,
                                                       T* __restrict__ y, int64_t rows, int N, float eps) {
  pdl_trigger();
  pdl_wait();
  constexpr int VN = 16 / sizeof(T);
  constexpr int R = MAXV <= 4 ? 2 : 1;
  int lane = threadIdx.x & 31;
  int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  int nv = N / VN;
  for (int64_t r0 = warp * R; r0 < rows; r0 += nwarps * R) {
    // the rows stay in registers in their stored form (4 registers per 16-byte
    // vector); each pass converts what it reads
    uint4 raw[R][MAXV];
    float s[R], q[R], mu[R], rs[R];
#pragma unroll
    for (int k = 0; k < R; k++) {
      s[k] = 0.f;
      const int64_t r = r0 + k;
#pragma unroll
      for (int t = 0; t < MAXV; t++) {
        int c = t * 32 + lane;
        if (c < nv && r < rows) {
          raw[k][t] = *(const uint4*)(x + r * N + (int64_t)c * VN);
          const T* e = (const T*)&raw[k][t];
#pragma unroll
          for (int j = 0; j < VN; j++) s[k] += to_f<T>(e[j]);
        } else {
          raw[k][t] = make_uint4(0u, 0u, 0u, 0u);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int k = 0; k < R; k++) s[k] += __shfl_xor_sync(0xffffffffu, s[k], o);
#pragma unroll
    for (int k = 0; k < R; k++) {
      mu[k] = s[k] / N;
      q[k] = 0.f;
#pragma unroll
      for (int t = 0; t < MAXV; t++) {
        if (t * 32 + lane < nv) {
          const T* e = (const T*)&raw[k][t];
#pragma unroll
          for (int j = 0; j < VN; j++) {
            float d = to_f<T>(e[j]) - mu[k];
            q[k] += d * d;
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int k = 0; k < R; k++) q[k] += __shfl_xor_sync(0xffffffffu, q[k], o);
#pragma unroll
    for (int k = 0; k < R; k++) rs[k] = rsqrtf(q[k] / N + eps);
#pragma unroll
    for (int t = 0; t < MAXV; t++) {
      int c = t * 32 + lane;
      if (c < nv) {
        uint4 out[R];
#pragma unroll
        for (int j = 0; j < VN; j += 4) {  // weight and bias four at a time (fewer live registers)
          const float4 a4 = ld_w4<WT>(w, c * VN + j, 1.f);
          const float4 b4 = ld_w4<WT>(b, c * VN + j, 0.f);
          const float wv[4] = {a4.x, a4.y, a4.z, a4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
          for (int k = 0; k < R; k++) {
            const T* e = (const T*)&raw[k][t];
            T* f = (T*)&out[k];
#pragma unroll
            for (int i = 0; i < 4; i++) {
              const float o = (to_f<T>(e[j + i]) - mu[k]) * rs[k] * wv[i] + bv[i];
              if constexpr (sizeof(T) == 4) ((float*)f)[j + i] = o;
              else if constexpr (std::is_same<T, __half>::value) f[j + i] = __float2half_rn(o);
              else f[j + i] = __float2bfloat16_rn(o);
            }
          }
        }
#pragma unroll
        for (int k = 0; k < R; k++)
          if (r0 + k < rows) *(uint4*)(y + (r0 + k) * N + (int64_t)c * VN) = out[k];
      }
    }
  }
}

// Rows longer than one warp's register tile: one 256-thread block per row (rows
// taken in turn by the grid), each thread holding up to MAXV 16-byte vectors;
// the mean and the centred sum of squares go through warp shuffles and the 8
// warps' partials in shared memory (read by every thread in the same order).
template <typename T, int MAXV, typename WT = float>
__global__ void __launch_bounds__(256) k_layernorm_blk(const T* __restrict__ x, const WT* __restrict__ w, const WT* __restrict__ b,
                                                       T* __restrict__ y, int64_t rows, int N, float eps) {
  pdl_trigger();
  pdl_wait();
  constexpr int VN = 16 / sizeof(T);
  __shared__ float sm[8];
  const int nv = N / VN;
  auto bsum = [&](float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = sm[0];
#pragma unroll
    for (int k = 1; k < 8; k++) t += sm[k];
    __syncthreads();
    return t;
  };
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    float v[MAXV][VN];
    float s = 0.f;
#pragma unroll
    for (int t = 0; t < MAXV; t++) {
      const int c = t * 256 + threadIdx.x;
      if (c < nv) {
        const uint4 raw = *(const uint4*)(x + r * N + (int64_t)c * VN);
        const T* e = (const T*)&raw;
#pragma unroll
        for (int j = 0; j < VN; j++) {
          v[t][j] = to_f<T>(e[j]);
          s += v[t][j];
        }
      }
    }
    const float mu = bsum(s) / N;
    float q = 0.f;
#pragma unroll
    for (int t = 0; t < MAXV; t++)
      if (t * 256 + (int)threadIdx.x < nv)
#pragma unroll
        for (int j = 0; j < VN; j++) {
          const float d = v[t][j] - mu;
          q += d * d;
        }
    const float rs = rsqrtf(bsum(q) / N + eps);
#pragma unroll
    for (int t = 0; t < MAXV; t++) {
      const int c = t * 256 + threadIdx.x;
      if (c < nv) {
        uint4 raw;
        T* e = (T*)&raw;
#pragma unroll
        for (int j = 0; j < VN; j += 4) {
          const float4 a4 = ld_w4<WT>(w, c * VN + j, 1.f);
          const float4 b4 = ld_w4<WT>(b, c * VN + j, 0.f);
          const float wv[4] = {a4.x, a4.y, a4.z, a4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
          for (int k = 0; k < 4; k++) {
            const float o = (v[t][j + k] - mu) * rs * wv[k] + bv[k];
            if constexpr (sizeof(T) == 4) ((float*)e)[j + k] = o;
            else if constexpr (std::is_same<T, __half>::value) e[j + k] = __float2half_rn(o);
            else e[j + k] = __float2bfloat16_rn(o);
          }
        }
        *(uint4*)(y + r * N + (int64_t)c * VN) = raw;
      }
    }
  }
}
template <typename T, typename WT = float>
void launch_layernorm_blk(const T* x, const WT* w, const WT* b, T* y, int64_t rows, int N, float eps, cudaStream_t st) {
  constexpr int VN = 16 / sizeof(T);
  const int per = (N / VN + 255) / 256;
  const unsigned blocks = (unsigned)std::min<int64_t>(rows, (int64_t)lc::num_sms() * 8);
  switch (per <= 1 ? 1 : per <= 2 ? 2 : per <= 4 ? 4 : 8) {
    case 1: lc::launch_chain(k_layernorm_blk<T, 1, WT>, dim3(blocks), dim3(256), 0, st, x, w, b, y, rows, N, eps); break;
    case 2: lc::launch_chain(k_layernorm_blk<T, 2, WT>, dim3(blocks), dim3(256), 0, st, x, w, b, y, rows, N, eps); break;
    case 4: lc::launch_chain(k_layernorm_blk<T, 4, WT>, dim3(blocks), dim3(256), 0, st, x, w, b, y, rows, N, eps); break;
    default: lc::launch_chain(k_layernorm_blk<T, 8, WT>, dim3(blocks), dim3(256), 0, st, x, w, b, y, rows, N, eps); break;
  }
}

// The register tile is sized to the row (vectors per lane = ceil(N / VN / 32)) so
// that short rows (H = 768 -> 3 vectors) keep full occupancy.
template <typename T, typename WT = float>
void launch_layernorm_vec(const T* x, const WT* w, const WT* b, T* y, int64_t rows, int N, float eps, cudaStream_t st) {
  constexpr int VN = 16 / sizeof(T);
  int per = (N / VN + 31) / 32;
  unsigned blocks = lc::blocks_for((per <= 4 ? (rows + 1) / 2 : rows) * 32, 256);  // two rows per warp for short rows
  switch (per) {
    case 0: case 1: lc::launch_chain(k_layernorm_vec<T, 1, WT>, dim3(blocks), dim3(256), 0, st, x, w, b, y, rows, N, eps); break;
    case 2: lc::launch_chain(k_layernorm_vec<T, 2, WT>, dim3(blocks), dim3(256), 0, st, x, w, b, y, rows, N, eps); break;
    case 3: lc::launch_chain(k_layernorm_vec<T, 3, WT>, dim3(blocks), dim3(256), 0, st, x, w, b, y, rows, N, eps); break;
    case 4: lc::launch_chain(k_layernorm_vec<T, 4, WT>, dim3(blocks), dim3(256), 0, st, x, w, b, y, rows, N, eps); break;
    case 5: case 6: lc::launch_chain(k_layernorm_vec<T, 6, WT>, dim3(blocks), dim3(256), 0, st, x, w, b, y, rows, N, eps); break;
    case 7: case 8: lc::launch_chain(k_layernorm_vec<T, 8, WT>, dim3(blocks), dim3(256), 0, st, x, w, b, y, rows, N, eps); break;
    default: lc::launch_chain(k_layernorm_vec<T, 12, WT>, dim3(blocks), dim3(256), 0, st, x, w, b, y, rows, N, eps); break;
  }
}

namespace lc {
// Dense f16/bf16 rows of N (N % 8 == 0, N <= 2048), f32 weight (or null), 16-byte aligned.
void layernorm_raw(const void* x, const float* w, void* y, int64_t rows, int N, float eps, int dtype, cudaStream_t st) {
  LC_CHECK(N % 8 == 0 && N <= 2048, "layernorm_raw: row length must be a multiple of 8, at most 2048");
  if (dtype == LC_F16)
    launch_layernorm_vec<__half, float>((const __half*)x, w, nullptr, (__half*)y, rows, N, eps, st);
  else
    launch_layernorm_vec<__nv_bfloat16, float>((const __nv_bfloat16*)x, w, nullptr, (__nv_bfloat16*)y, rows, N, eps, st);
  LC_LAUNCHED(1);
}
}  // namespace lc

template <typename CT>
__global__ void k_layernorm_generic(const char* x, int xdt, const char* w, int wdt, const char* b, int bdt, char* y, int ydt,
                                    int64_t rows, int64_t N, double eps) {
  int lane = threadIdx.x & 31;
  int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += nwarps) {
    CT s = 0;
    for (int64_t j = lane; j < N; j += 32) s += ld_as<CT>(x, xdt, r * N + j);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    CT mu = s / (CT)N;
    CT q = 0;
    for (int64_t j = lane; j < N; j += 32) {
      CT d = ld_as<CT>(x, xdt, r * N + j) - mu;
      q += d * d;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    CT rs = (CT)1 / sqrt(q / (CT)N + (CT)eps);
    for (int64_t j = lane; j < N; j += 32) {
      CT o = (ld_as<CT>(x, xdt, r * N + j) - mu) * rs;
      if (w) o *= ld_as<CT>(w, wdt, j);
      if (b) o += ld_as<CT>(b, bdt, j);
      st_as<CT>(y, ydt, r * N + j, o);
    }
  }
}

// ------------------------------------------------------------- gathers

// out row r = table[ids[r]] (zeros for an out-of-range id)
__global__ void k_gather_rows(const char* table, int64_t V, int64_t rowbytes, const char* ids, int iddt, char* out, int64_t n,
                              int64_t group, const int64_t group_rows) {
  pdl_trigger();
  pdl_wait();
  // group/group_rows: for gatherRows, row r reads from batch r / group, offset batch*group_rows
  int lane = threadIdx.x & 31;
  int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  bool vec = (rowbytes % 16 == 0) && (((uintptr_t)table & 15) == 0) && (((uintptr_t)out & 15) == 0);
  for (int64_t r = warp; r < n; r += nwarps) {
    int64_t id = ld_as<int64_t>(ids, iddt, r);
    int64_t base = group > 0 ? (r / group) * group_rows : 0;
    bool ok = id >= 0 && id < V;
    const char* src = table + (base + (ok ? id : 0)) * rowbytes;
    char* dst = out + r * rowbytes;
    if (vec) {
      for (int64_t c = lane; c < rowbytes / 16; c += 32)
        ((uint4*)dst)[c] = ok ? ((const uint4*)src)[c] : make_uint4(0, 0, 0, 0);
    } else {
      for (int64_t c = lane; c < rowbytes; c += 32) dst[c] = ok ? src[c] : 0;
    }
  }
}

// ------------------------------------------------------------- rope
// index.ts:225-229: split-half rotation over x [..., L, D], positions 0..L-1.
// cos/sin come from a table built on the host with MLX's f32 angle rounding
// (packages/backend-webgpu/src/backend.ts:1179-1195).

__global__ void k_rope(TV x, const float* __restrict__ cs, int64_t rows, int64_t L, int half, int cap, char* out) {
  // cs: [cap, half] cos then [cap, half] sin
  LC_GRID_STRIDE(t, rows * half) {
    int64_t r = t / half;
    int i = (int)(t % half);
    int64_t l = r % L;
    // offset of row r (dims 0..ndim-2) in x
    int64_t rr = r, off = 0;
    for (int d = x.ndim - 2; d >= 0; d--) {
      off += (rr % x.shape[d]) * x.strides[d];
      rr /= x.shape[d];
    }
    int64_t sd = x.strides[x.ndim - 1];
    float a = ld_as<float>(x.ptr, x.dtype, off + i * sd);
    float b = ld_as<float>(x.ptr, x.dtype, off + (i + half) * sd);
    float c = cs[l * half + i], s = cs[(int64_t)cap * half + l * half + i];
    int64_t o = r * 2 * half;
    st_as<float>(out, x.dtype, o + i, a * c - b * s);
    st_as<float>(out, x.dtype, o + i + half, b * c + a * s);
  }
}

// Vectorised path: last dimension dense, half a multiple of 4, rows 4-element
// aligned. One thread per 4 pairs (i, i + half): two 4-element loads, the
// cos / sin quads of the position, two 4-element stores; 32-bit index math.
template <typename T>
__global__ void __launch_bounds__(256) k_rope_vec(TV x, const float* __restrict__ cs, int rows, int L, int half, int cap, T* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int qpr = half / 4;
  const int64_t n = (int64_t)rows * qpr;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(t / qpr), i = (int)(t % qpr) * 4;
    const int l = r % L;
    int64_t off = 0;
    int rr = r;
    for (int d = x.ndim - 2; d >= 0; d--) {
      const int sh = (int)x.shape[d];
      off += (int64_t)(rr % sh) * x.strides[d];
      rr /= sh;
    }
    const T* p = (const T*)x.ptr + off + i;
    float a[4], b[4];
    if constexpr (sizeof(T) == 4) {
      const float4 va = *(const float4*)p, vb = *(const float4*)(p + half);
      a[0] = va.x, a[1] = va.y, a[2] = va.z, a[3] = va.w;
      b[0] = vb.x, b[1] = vb.y, b[2] = vb.z, b[3] = vb.w;
    } else {
      const uint2 ua = *(const uint2*)p, ub = *(const uint2*)(p + half);
      const T* ha = (const T*)&ua;
      const T* hb = (const T*)&ub;
#pragma unroll
      for (int j = 0; j < 4; j++) a[j] = to_f(ha[j]), b[j] = to_f(hb[j]);
    }
    const float4 c = __ldg((const float4*)(cs + (int64_t)l * half + i));
    const float4 sn = __ldg((const float4*)(cs + (int64_t)cap * half + (int64_t)l * half + i));
    const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {sn.x, sn.y, sn.z, sn.w};
    T* o = out + (int64_t)r * 2 * half + i;
    T ya[4], yb[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      ya[j] = from_f<T>(a[j] * cc[j] - b[j] * ss[j]);
      yb[j] = from_f<T>(b[j] * cc[j] + a[j] * ss[j]);
    }
    if constexpr (sizeof(T) == 4) {
      *(float4*)o = *(const float4*)ya;
      *(float4*)(o + half) = *(const float4*)yb;
    } else {
      *(uint2*)o = *(const uint2*)ya;
      *(uint2*)(o + half) = *(const uint2*)yb;
    }
  }
}

// 16-bit rows with half % 8 == 0, rows 8-element strided and 16-byte aligned:
// one thread per 8 pairs, 16-byte loads and stores of x and y, the position's
// cos / sin as four float4 loads. The row offset is split into the row's
// position l (fastest) and the rows above it, whose offsets a table of the
// leading dims' strides gives with at most two divisions.
template <typename T>
__global__ void __launch_bounds__(256) k_rope_vec8(TV x, const float* __restrict__ cs, int rows, int L, int half, int cap, T* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int qpr = half / 8;
  const int64_t n = (int64_t)rows * qpr;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(t / qpr), i = (int)(t % qpr) * 8;
    const int l = r % L;
    int64_t off = (int64_t)l * x.strides[x.ndim - 2];
    int rr = r / L;
    for (int d = x.ndim - 3; d >= 0; d--) {
      const int sh = (int)x.shape[d];
      off += (int64_t)(rr % sh) * x.strides[d];
      rr /= sh;
    }
    const T* p = (const T*)x.ptr + off + i;
    const uint4 ua = *(const uint4*)p, ub = *(const uint4*)(p + half);
    const T* ha = (const T*)&ua;
    const T* hb = (const T*)&ub;
    const float4* cp = (const float4*)(cs + (int64_t)l * half + i);
    const float4* sp = (const float4*)(cs + (int64_t)cap * half + (int64_t)l * half + i);
    const float4 c0 = __ldg(cp), c1 = __ldg(cp + 1), s0 = __ldg(sp), s1 = __ldg(sp + 1);
    const float cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float ss[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    uint4 ra, rb;
    T* ya = (T*)&ra;
    T* yb = (T*)&rb;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const float a = to_f(ha[j]), b = to_f(hb[j]);
      ya[j] = from_f<T>(a * cc[j] - b * ss[j]);
      yb[j] = from_f<T>(b * cc[j] + a * ss[j]);
    }
    T* o = out + (int64_t)r * 2 * half + i;
    *(uint4*)o = ra;
    *(uint4*)(o + half) = rb;
  }
}

namespace {
struct RopeTable {
  float* d = nullptr;
  int cap = 0;
};
std::map<std::tuple<int, double, bool>, RopeTable>& rope_cache() {
  static std::map<std::tuple<int, double, bool>, RopeTable> m;
  return m;
}
// Outgrown tables stay allocated until the caches are destroyed: a recorded
// CUDA graph (Backend.compile) keeps the pointer it was captured with.
std::vector<float*>& rope_retired() {
  static std::vector<float*> v;
  return v;
}
}  // namespace

namespace lc {
// cos/sin table (f32) for head dim D and `base`, cap >= L positions:
// [cap][half] cos ++ [cap][half] sin, or with position_minor the GEMM
// epilogue's layout [half/2][cap] of float4 (cos 2i, cos 2i+1, sin 2i,
// sin 2i+1): a warp's 32 rows are (mostly) consecutive positions, so each
// 16-byte load of the warp reads one contiguous run.
const float* rope_table(int D, double base, int L, int* cap_out, bool position_minor) {
  auto& t = rope_cache()[{D, base, position_minor}];
  if (t.cap < L) {
    int cap = 64;
    while (cap < L) cap <<= 1;
    int half = D / 2;
    std::vector<float> h((size_t)2 * cap * half);
    float lb = (float)std::log2(base);
    for (int i = 0; i < half; i++) {
      float e = (float)(-(double)(float)((double)i / half) * (double)lb);
      float inv = (float)std::pow(2.0, (double)e);
      for (int l = 0; l < cap; l++) {
        float th = (float)((double)l * (double)inv);
        if (position_minor) {
          const size_t base = ((size_t)(i / 2) * cap + l) * 4 + (i & 1);
          h[base] = (float)std::cos((double)th);
          h[base + 2] = (float)std::sin((double)th);
        } else {
          const size_t ci = (size_t)l * half + i;
          h[ci] = (float)std::cos((double)th);
          h[(size_t)cap * half + ci] = (float)std::sin((double)th);
        }
      }
    }
    if (t.d) rope_retired().push_back(t.d);
    CUDA_OK(cudaMalloc(&t.d, h.size() * sizeof(float)));
    CUDA_OK(cudaMemcpy(t.d, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice));
    t.cap = cap;
  }
  *cap_out = t.cap;
  return t.d;
}
}  // namespace lc

void lc_internal_destroy_caches() {
  for (auto& kv : rope_cache())
    if (kv.second.d) cudaFree(kv.second.d);
  rope_cache().clear();
  for (float* d : rope_retired()) cudaFree(d);
  rope_retired().clear();
  lc_gemm_destroy_caches();
}

// ------------------------------------------------------------- sdpa (generic)
// index.ts:230-237. One warp per query row; keys in chunks of 32 with an
// online softmax in f32. Any dtype/strides, D and Dv <= 256, bool mask
// broadcast to [B, H, Lq, Lk] (strides 0 on broadcast axes).

#define SDPA_MAXD 256
__global__ void __launch_bounds__(128) k_sdpa_generic(TV q, TV k, TV v, TV m, int has_mask, float scale, char* out, int odt,
                                                      int64_t B, int64_t H, int64_t Lq, int64_t Lk, int D, int Dv) {
  __shared__ float qs[4][SDPA_MAXD];
  int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int64_t row = (int64_t)blockIdx.x * 4 + w;
  if (row >= B * H * Lq) return;
  int64_t i = row % Lq, bh = row / Lq, h = bh % H, b = bh / H;
  int64_t qo = b * q.strides[0] + h * q.strides[1] + i * q.strides[2];
  for (int d = lane; d < D; d += 32) qs[w][d] = ld_as<float>(q.ptr, q.dtype, qo + d * q.strides[3]) * scale;
  __syncwarp();
  int64_t kb = b * k.strides[0] + h * k.strides[1];
  int64_t vb = b * v.strides[0] + h * v.strides[1];
  int64_t mb = has_mask ? b * m.strides[0] + h * m.strides[1] + i * m.strides[2] : 0;
  float acc[SDPA_MAXD / 32];
#pragma unroll
  for (int t = 0; t < SDPA_MAXD / 32; t++) acc[t] = 0.f;
  float mx = -INFINITY, l = 0.f;
  for (int64_t j0 = 0; j0 < Lk; j0 += 32) {
    int64_t j = j0 + lane;
    float s = -INFINITY;
    if (j < Lk) {
      bool keep = true;
      if (has_mask) keep = ((const uint8_t*)m.ptr)[mb + j * m.strides[3]] != 0;
      if (keep) {
        float dot = 0.f;
        int64_t ko = kb + j * k.strides[2];
        for (int d = 0; d < D; d++) dot += qs[w][d] * ld_as<float>(k.ptr, k.dtype, ko + d * k.strides[3]);
        s = dot;
      }
    }
    float cm = s;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
    float nm = fmaxf(mx, cm);
    if (nm == -INFINITY) continue;  // every key so far masked
    float corr = __expf(mx - nm);
    float p = (s == -INFINITY) ? 0.f : __expf(s - nm);
    float ps = p;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
    l = l * corr + ps;
#pragma unroll
    for (int t = 0; t < SDPA_MAXD / 32; t++) acc[t] *= corr;
    int cnt = (Lk - j0) < 32 ? (int)(Lk - j0) : 32;
    for (int jj = 0; jj < cnt; jj++) {
      float pj = __shfl_sync(0xffffffffu, p, jj);
      if (pj == 0.f) continue;
      int64_t vo = vb + (j0 + jj) * v.strides[2];
#pragma unroll
      for (int t = 0; t < SDPA_MAXD / 32; t++) {
        int d = t * 32 + lane;
        if (d < Dv) acc[t] += pj * ld_as<float>(v.ptr, v.dtype, vo + d * v.strides[3]);
      }
    }
    mx = nm;
  }
  float inv = 1.f / l;
  int64_t oo = row * Dv;
#pragma unroll
  for (int t = 0; t < SDPA_MAXD / 32; t++) {
    int d = t * 32 + lane;
    if (d < Dv) st_as<float>(out, odt, oo + d, acc[t] * inv);
  }
}

// ------------------------------------------------------------- geglu / meanPool

template <typename T>
__global__ void __launch_bounds__(256) k_geglu_vec(const T* __restrict__ x, T* __restrict__ y, int64_t rows, int64_t F) {
  pdl_trigger();
  pdl_wait();
  constexpr int VN = 16 / sizeof(T);
  int64_t nv = F / VN;
  LC_GRID_STRIDE(t, rows * nv) {
    int64_t r = t / nv, c = (t % nv) * VN;
    uint4 ra = *(const uint4*)(x + r * 2 * F + c);
    uint4 rb = *(const uint4*)(x + r * 2 * F + F + c);
    uint4 ro;
    const T* a = (const T*)&ra;
    const T* g = (const T*)&rb;
    T* o = (T*)&ro;
    if constexpr (sizeof(T) == 4) {
#pragma unroll
      for (int j = 0; j < VN; j++) {
        const float av = ((const float*)a)[j], gv = ((const float*)g)[j];
        ((float*)o)[j] = 0.5f * av * (1.0f + erff(av * 0.7071067811865476f)) * gv;
      }
    } else {
      // stored in 16 bits: erf by Abramowitz & Stegun 7.1.26 (|error| <= 1.5e-7), packed pairs
#pragma unroll
      for (int j = 0; j < VN; j += 2) {
        float2 av, gv;
        if constexpr (std::is_same<T, __half>::value) {
          av = __half22float2(*(const __half2*)(a + j));
          gv = __half22float2(*(const __half2*)(g + j));
          const float2 r = mul2(gelu_as2(av), gv);
          *(__half2*)(o + j) = __floats2half2_rn(r.x, r.y);
        } else {
          av = __bfloat1622float2(*(const __nv_bfloat162*)(a + j));
          gv = __bfloat1622float2(*(const __nv_bfloat162*)(g + j));
          const float2 r = mul2(gelu_as2(av), gv);
          *(__nv_bfloat162*)(o + j) = __floats2bfloat162_rn(r.x, r.y);
        }
      }
    }
    *(uint4*)(y + r * F + c) = ro;
  }
}

template <typename CT>
__global__ void k_geglu_generic(const char* x, int xdt, char* y, int ydt, int64_t rows, int64_t F) {
  LC_GRID_STRIDE(t, rows * F) {
    int64_t r = t / F, c = t % F;
    CT a = ld_as<CT>(x, xdt, r * 2 * F + c), g = ld_as<CT>(x, xdt, r * 2 * F + F + c);
    st_as<CT>(y, ydt, t, (CT)0.5 * a * ((CT)1 + erf(a * (CT)0.7071067811865476)) * g);
  }
}

// Dense f16 / bf16 / f32 x with D % (16 / sizeof(T)) == 0: block (32*VEC-column
// chunk, b, slice of 256 positions); each of its 8 warps takes one 32-row
// chunk of the slice: it reads the chunk's 32 mask entries at once (one per
// lane, a ballot gives the kept rows), then each lane sums VEC columns of the
// kept rows from 16-byte loads, eight rows in flight; the warps' partial sums
// and counts combine in shared memory. With one slice (L <= 256) the block
// writes the mean; otherwise it writes its slice's sums and count and
// k_mean_pool_fin adds the slices in order.
template <typename T>
__global__ void __launch_bounds__(256) k_mean_pool_vec(const T* __restrict__ x, const char* mask, int mdt, float* __restrict__ out,
                                                       float* __restrict__ part, float* __restrict__ pcnt, int64_t L, int64_t D) {
  pdl_trigger();
  pdl_wait();
  constexpr int VEC = 16 / sizeof(T);
  constexpr int UNR = 8;
  __shared__ float sp[8][32 * VEC];
  __shared__ float cnt[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t b = blockIdx.y, B = gridDim.y, z = blockIdx.z;
  const int64_t c0 = (int64_t)blockIdx.x * 32 * VEC + lane * VEC;
  const bool on = c0 < D;
  float acc[VEC];
#pragma unroll
  for (int j = 0; j < VEC; j++) acc[j] = 0.f;
  const int64_t l0 = z * 256 + (int64_t)warp * 32;
  const bool keep = l0 + lane < L && ld_as<int64_t>(mask, mdt, b * L + l0 + lane) != 0;
  const uint32_t bits = __ballot_sync(0xffffffffu, keep);
  const float n = (float)__popc(bits);
  if (on) {
#pragma unroll 1
    for (int i0 = 0; i0 < 32; i0 += UNR) {
      if (((bits >> i0) & ((1u << UNR) - 1u)) == 0u) continue;  // warp-uniform
      uint4 raw[UNR];
#pragma unroll
      for (int u = 0; u < UNR; u++)
        raw[u] = (bits >> (i0 + u)) & 1u ? *(const uint4*)(x + (b * L + l0 + i0 + u) * D + c0) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int u = 0; u < UNR; u++) {
        const T* e = (const T*)&raw[u];
#pragma unroll
        for (int j = 0; j < VEC; j++) acc[j] += to_f<T>(e[j]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < VEC; j++) sp[warp][lane * VEC + j] = acc[j];
  if (lane == 0) cnt[warp] = n;
  __syncthreads();
  if (warp == 0) {
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; w++) tot += cnt[w];
    const float inv = 1.f / fmaxf(tot, 1.f);
    if (on)
#pragma unroll
      for (int j = 0; j < VEC; j++) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) s += sp[w][lane * VEC + j];
        if (gridDim.z == 1) out[b * D + c0 + j] = s * inv;
        else part[(z * B + b) * D + c0 + j] = s;
      }
    if (gridDim.z > 1 && blockIdx.x == 0 && lane == 0) pcnt[z * B + b] = tot;
  }
}

// The slices' sums of k_mean_pool_vec added in slice order, divided by the count.
__global__ void __launch_bounds__(256) k_mean_pool_fin(const float* __restrict__ part, const float* __restrict__ pcnt, float* __restrict__ out,
                                                       int64_t B, int64_t D, int LS) {
  pdl_trigger();
  pdl_wait();
  LC_GRID_STRIDE(t, B * D) {
    const int64_t b = t / D, d = t % D;
    float s = 0.f, n = 0.f;
    for (int z = 0; z < LS; z++) {
      s += part[(z * B + b) * D + d];
      n += pcnt[z * B + b];
    }
    out[t] = s / fmaxf(n, 1.f);
  }
}

__global__ void k_mean_pool(const char* x, int xdt, const char* mask, int mdt, float* out, int64_t B, int64_t L, int64_t D) {
  LC_GRID_STRIDE(t, B * D) {
    int64_t b = t / D, d = t % D;
    float s = 0.f, n = 0.f;
    for (int64_t l = 0; l < L; l++) {
      if (ld_as<int64_t>(mask, mdt, b * L + l) != 0) {
        s += ld_as<float>(x, xdt, (b * L + l) * D + d);
        n += 1.f;
      }
    }
    out[t] = s / fmaxf(n, 1.f);
  }
}

// ------------------------------------------------------------- matmul / SIMT linear

// C[b] = A[b] (m x k) · B[b] (k x n) (B given by strides so w[N,K] works as Bᵀ),
// 64x64 tiles, 16-deep k steps, 4x4 outputs per thread, CT accumulation.
struct MM {
  const char* a;
  const char* b;
  char* c;
  const char* bias;
  int adt, bdt, cdt, biasdt;
  int64_t m, n, k;
  int64_t sam, sak, sbk, sbn;  // element strides inside one matrix
  // batch addressing: up to 6 batch dims, broadcast strides for a and b
  int nb;
  int64_t bshape[6], bsa[6], bsb[6];
};

template <typename CT>
__global__ void __launch_bounds__(256) k_matmul(MM p) {
  __shared__ CT As[16][64 + 1];
  __shared__ CT Bs[16][64 + 1];
  int64_t bz = blockIdx.z;
  int64_t offa = 0, offb = 0, rem = bz;
  for (int d = p.nb - 1; d >= 0; d--) {
    int64_t c = rem % p.bshape[d];
    rem /= p.bshape[d];
    offa += c * p.bsa[d];
    offb += c * p.bsb[d];
  }
  int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  int64_t m0 = (int64_t)blockIdx.y * 64, n0 = (int64_t)blockIdx.x * 64;
  CT acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0;
  for (int64_t k0 = 0; k0 < p.k; k0 += 16) {
    for (int e = threadIdx.x; e < 16 * 64; e += 256) {
      int kk = e % 16, mm = e / 16;
      int64_t gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < p.m && gk < p.k) ? ld_as<CT>(p.a, p.adt, offa + gm * p.sam + gk * p.sak) : (CT)0;
      int nn = e / 16;
      int64_t gn = n0 + nn;
      Bs[kk][nn] = (gn < p.n && gk < p.k) ? ld_as<CT>(p.b, p.bdt, offb + gk * p.sbk + gn * p.sbn) : (CT)0;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; kk++) {
      CT av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; i++) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; j++) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] += av[i] * bv[j];
    }
    __syncthreads();
  }
  int64_t offc = (int64_t)bz * p.m * p.n;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    int64_t gm = m0 + ty * 4 + i;
    if (gm >= p.m) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      int64_t gn = n0 + tx * 4 + j;
      if (gn >= p.n) continue;
      CT v = acc[i][j];
      if (p.bias) v += ld_as<CT>(p.bias, p.biasdt, gn);
      st_as<CT>(p.c, p.cdt, offc + gm * p.n + gn, v);
    }
  }
}

// y[m, n] = x[m, :] · w[n, :] (+ bias[n]) for few rows: one warp per output,
// lanes striding over K, f32 accumulation (the contract's, index.ts:211-215).
// The 64 x 64-tile SIMT kernel would put only ceil(N/64) blocks on the GPU.
__global__ void __launch_bounds__(256) k_linear_rows(const char* x, int xdt, const char* w, int wdt, const char* bias, int bdt, char* y,
                                                     int ydt, int64_t M, int64_t N, int64_t K) {
  pdl_trigger();
  pdl_wait();
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= M * N) return;
  const int64_t m = warp / N, n = warp % N;
  float acc = 0.f;
  for (int64_t k = lane; k < K; k += 32) acc = fmaf(ld_as<float>(x, xdt, m * K + k), ld_as<float>(w, wdt, n * K + k), acc);
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) {
    if (bias) acc += ld_as<float>(bias, bdt, n);
    st_as<float>(y, ydt, m * N + n, acc);
  }
}

// The same for dense 16-bit x and w rows with K % VW == 0 and rows aligned to
// VW elements (VW = 8: 16-byte loads; 4: 8-byte loads, e.g. K = 772), the
// whole K range of a lane in flight at once.
template <typename T, int VW>
__global__ void __launch_bounds__(256) k_linear_rows16(const T* __restrict__ x, const T* __restrict__ w, const char* bias, int bdt, char* y,
                                                       int ydt, int M, int N, int K) {
  pdl_trigger();
  pdl_wait();
  using V = typename std::conditional<VW == 8, uint4, uint2>::type;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= (int64_t)M * N) return;
  const int m = (int)(warp / N), n = (int)(warp % N);
  const V* xr = (const V*)(x + (int64_t)m * K);
  const V* wr = (const V*)(w + (int64_t)n * K);
  const int nv = K / VW;
  float acc = 0.f;
#pragma unroll 4
  for (int v = lane; v < nv; v += 32) {
    const V a = __ldg(xr + v), b = __ldg(wr + v);
    const T* ae = (const T*)&a;
    const T* be = (const T*)&b;
#pragma unroll
    for (int j = 0; j < VW; j++) acc = fmaf(to_f<T>(ae[j]), to_f<T>(be[j]), acc);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) {
    if (bias) acc += ld_as<float>(bias, bdt, n);
    st_as<float>(y, ydt, (int64_t)m * N + n, acc);
  }
}

namespace {

void launch_mm(const MM& p, int64_t batch, bool dbl) {
  dim3 grid((unsigned)((p.n + 63) / 64), (unsigned)((p.m + 63) / 64), (unsigned)batch);
  LC_CHECK(batch <= 65535 && grid.y <= 65535, "matmul: batch or row count too large for the SIMT path");
  if (dbl) k_matmul<double><<<grid, 256, 0, stream()>>>(p);
  else k_matmul<float><<<grid, 256, 0, stream()>>>(p);
  LC_LAUNCHED(1);
}

int float_out(int a, int b) {
  int d = promote(a, b);
  return is_float(d) ? d : LC_F32;
}

}  // namespace

namespace lc {
// y [M, N] = x [M, K] · w[N, K]ᵀ (+ bias) on the SIMT path (exact f32 / f64 accumulation).
void linear_simt(const LcTensor* x2, const LcTensor* w, const LcTensor* bias, LcTensor* y) {
  MM p{};
  p.a = x2->data(); p.adt = x2->dtype;
  p.b = w->data(); p.bdt = w->dtype;
  p.c = y->data(); p.cdt = y->dtype;
  p.bias = bias ? bias->data() : nullptr; p.biasdt = bias ? bias->dtype : 0;
  p.m = x2->shape[0]; p.k = x2->shape[1]; p.n = w->shape[0];
  p.sam = p.k; p.sak = 1;
  p.sbk = 1; p.sbn = p.k;  // w[n, k]
  p.nb = 0;
  const bool dbl = y->dtype == LC_F64 || x2->dtype == LC_F64 || w->dtype == LC_F64;
  if (p.m && p.n && p.m <= 16 && !dbl && p.m * p.n < ((int64_t)1 << 26)) {
    const unsigned blocks = (unsigned)((p.m * p.n * 32 + 255) / 256);
    const bool h16 = is_half(x2->dtype) && w->dtype == x2->dtype && p.k < INT32_MAX;
    const int vw = !h16 ? 0 : (p.k % 8 == 0 && (((uintptr_t)p.a | (uintptr_t)p.b) & 15) == 0) ? 8
                            : (p.k % 4 == 0 && (((uintptr_t)p.a | (uintptr_t)p.b) & 7) == 0) ? 4 : 0;
#define LC_ROWS16(T, VW)                                                                                                               \
  lc::launch_chain(k_linear_rows16<T, VW>, dim3(blocks), dim3(256), 0, stream(), (const T*)p.a, (const T*)p.b, p.bias, p.biasdt, p.c, \
                   p.cdt, (int)p.m, (int)p.n, (int)p.k)
    if (vw == 8 && x2->dtype == LC_F16) LC_ROWS16(__half, 8);
    else if (vw == 8) LC_ROWS16(__nv_bfloat16, 8);
    else if (vw == 4 && x2->dtype == LC_F16) LC_ROWS16(__half, 4);
    else if (vw == 4) LC_ROWS16(__nv_bfloat16, 4);
#undef LC_ROWS16
    else
      lc::launch_chain(k_linear_rows, dim3(blocks), dim3(256), 0, stream(), p.a, p.adt, p.b, p.bdt, p.bias, p.biasdt, p.c, p.cdt, p.m,
                       p.n, p.k);
    LC_LAUNCHED(1);
    return;
  }
  if (p.m && p.n) launch_mm(p, 1, dbl);
}
}  // namespace lc

extern "C" {

int lc_layer_norm(lc_tensor* out, lc_tensor xh, lc_tensor wh, lc_tensor bh, double eps) {
  LC_API_BEGIN
  LcTensor* x0 = check(xh, "layerNorm");
  LC_CHECK(x0->ndim >= 1, "layerNorm: scalar input");
  int64_t N = x0->shape[x0->ndim - 1];
  LcTensor* w0 = wh ? check(wh, "layerNorm weight") : nullptr;
  LcTensor* b0 = bh ? check(bh, "layerNorm bias") : nullptr;
  if (w0) LC_CHECK(w0->numel() == N, "layerNorm: weight size differs from the last axis");
  if (b0) LC_CHECK(b0->numel() == N, "layerNorm: bias size differs from the last axis");
  int odt = is_float(x0->dtype) ? x0->dtype : LC_F32;
  LcTensor* y = alloc(odt, x0->dims());
  int64_t rows = N ? x0->numel() / N : 0;
  if (rows) {
    LcTensor* x = contiguous(x0);
    // the vector kernel reads f32 weight/bias; convert others once (they are [N])
    auto as_f32 = [](LcTensor* t) -> LcTensor* {
      if (!t) return nullptr;
      if (t->dtype == LC_F32 && t->contiguous()) return t;
      LcTensor* f = alloc(LC_F32, {t->numel()});
      LcTensor* flat = view_of(t, {t->numel()}, {t->strides[t->ndim - 1]}, t->offset);
      copy_into(t->contiguous() ? flat : t, f);
      release(flat);
      return f;
    };
    bool f64 = x->dtype == LC_F64;
    // 16-bit rows with dense weight / bias of the same type are read as they are
    auto same16 = [&](LcTensor* t) { return !t || (t->dtype == x->dtype && t->contiguous()); };
    const bool w16 = is_half(x->dtype) && x->dtype == odt && same16(w0) && same16(b0) && (w0 || b0);
    LcTensor* w = (f64 || w16) ? w0 : as_f32(w0);
    LcTensor* b = (f64 || w16) ? b0 : as_f32(b0);
    const char* wp = w ? w->data() : nullptr;
    const char* bp = b ? b->data() : nullptr;
    int wdt = w ? w->dtype : 0, bdt = b ? b->dtype : 0;
    unsigned blocks = blocks_for(rows * 32, 256);
    cudaStream_t st = stream();
    bool aligned = (((uintptr_t)x->data() | (uintptr_t)y->data() | (uintptr_t)wp | (uintptr_t)bp) & 15) == 0;
    int vn = x->dtype == LC_F32 ? 4 : 8;
    bool vec = aligned && x->dtype == odt && (odt == LC_F32 || is_half(odt)) && N % vn == 0 && N / vn <= 32 * 12;
    bool blk = aligned && x->dtype == odt && (odt == LC_F32 || is_half(odt)) && N % vn == 0 && N / vn <= 256 * 8;
    const float* wf = (const float*)wp;
    const float* bf = (const float*)bp;
    if (w16 && (vec || blk)) {
      if (odt == LC_F16) {
        const __half *wh = (const __half*)wp, *bh = (const __half*)bp;
        if (vec) launch_layernorm_vec<__half, __half>((const __half*)x->data(), wh, bh, (__half*)y->data(), rows, (int)N, (float)eps, st);
        else launch_layernorm_blk<__half, __half>((const __half*)x->data(), wh, bh, (__half*)y->data(), rows, (int)N, (float)eps, st);
      } else {
        const __nv_bfloat16 *wh = (const __nv_bfloat16*)wp, *bh = (const __nv_bfloat16*)bp;
        if (vec)
          launch_layernorm_vec<__nv_bfloat16, __nv_bfloat16>((const __nv_bfloat16*)x->data(), wh, bh, (__nv_bfloat16*)y->data(), rows, (int)N,
                                                             (float)eps, st);
        else
          launch_layernorm_blk<__nv_bfloat16, __nv_bfloat16>((const __nv_bfloat16*)x->data(), wh, bh, (__nv_bfloat16*)y->data(), rows, (int)N,
                                                             (float)eps, st);
      }
    } else if (vec) {
      if (odt == LC_F16) launch_layernorm_vec<__half>((const __half*)x->data(), wf, bf, (__half*)y->data(), rows, (int)N, (float)eps, st);
      else if (odt == LC_BF16) launch_layernorm_vec<__nv_bfloat16>((const __nv_bfloat16*)x->data(), wf, bf, (__nv_bfloat16*)y->data(), rows, (int)N, (float)eps, st);
      else launch_layernorm_vec<float>((const float*)x->data(), wf, bf, (float*)y->data(), rows, (int)N, (float)eps, st);
    } else if (blk) {
      if (odt == LC_F16) launch_layernorm_blk<__half>((const __half*)x->data(), wf, bf, (__half*)y->data(), rows, (int)N, (float)eps, st);
      else if (odt == LC_BF16) launch_layernorm_blk<__nv_bfloat16>((const __nv_bfloat16*)x->data(), wf, bf, (__nv_bfloat16*)y->data(), rows, (int)N, (float)eps, st);
      else launch_layernorm_blk<float>((const float*)x->data(), wf, bf, (float*)y->data(), rows, (int)N, (float)eps, st);
    } else if (x->dtype == LC_F64) {
      k_layernorm_generic<double><<<blocks, 256, 0, st>>>(x->data(), x->dtype, wp, wdt, bp, bdt, y->data(), odt, rows, N, eps);
    } else {
      k_layernorm_generic<float><<<blocks, 256, 0, st>>>(x->data(), x->dtype, wp, wdt, bp, bdt, y->data(), odt, rows, N, eps);
    }
    LC_LAUNCHED(1);
    if (x != x0) release(x);
    if (w && w != w0) release(w);
    if (b && b != b0) release(b);
  }
  *out = handle(y);
  LC_API_END
}

int lc_embedding(lc_tensor* out, lc_tensor th, lc_tensor ih) {
  LC_API_BEGIN
  LcTensor* t0 = check(th, "embedding table");
  LcTensor* i0 = check(ih, "embedding ids");
  LC_CHECK(t0->ndim == 2, "embedding: table must be [V, D]");
  LC_CHECK(!is_float(i0->dtype), "embedding: ids must be an integer tensor");
  std::vector<int64_t> sh = i0->dims();
  sh.push_back(t0->shape[1]);
  LcTensor* y = alloc(t0->dtype, sh);
  int64_t n = i0->numel();
  if (n && t0->shape[1]) {
    LcTensor* t = contiguous(t0);
    LcTensor* ids = contiguous(i0);
    lc::launch_chain(k_gather_rows, dim3(blocks_for(n * 32, 256)), dim3(256), 0, stream(), t->data(), t->shape[0], t->shape[1] * dtype_size(t->dtype),
                                                                 ids->data(), ids->dtype, y->data(), n, 0, 0);
    LC_LAUNCHED(1);
    if (t != t0) release(t);
    if (ids != i0) release(ids);
  }
  *out = handle(y);
  LC_API_END
}

int lc_gather_rows(lc_tensor* out, lc_tensor xh, lc_tensor ih) {
  LC_API_BEGIN
  LcTensor* x0 = check(xh, "gatherRows x");
  LcTensor* i0 = check(ih, "gatherRows idx");
  LC_CHECK(x0->ndim == 3 && i0->ndim == 2 && i0->shape[0] == x0->shape[0], "gatherRows: x [B, L, D] and idx [B, M] expected");
  int64_t B = x0->shape[0], L = x0->shape[1], D = x0->shape[2], M = i0->shape[1];
  LcTensor* y = alloc(x0->dtype, {B, M, D});
  if (B * M && D) {
    LcTensor* x = contiguous(x0);
    LcTensor* ids = contiguous(i0);
    lc::launch_chain(k_gather_rows, dim3(blocks_for(B * M * 32, 256)), dim3(256), 0, stream(), x->data(), L, D * dtype_size(x->dtype), ids->data(), ids->dtype,
                                                                     y->data(), B * M, M, L);
    LC_LAUNCHED(1);
    if (x != x0) release(x);
    if (ids != i0) release(ids);
  }
  *out = handle(y);
  LC_API_END
}

int lc_rope(lc_tensor* out, lc_tensor xh, double base) {
  LC_API_BEGIN
  LcTensor* x = check(xh, "rope");
  LC_CHECK(x->ndim >= 2, "rope: x must be [..., L, D]");
  int64_t L = x->shape[x->ndim - 2], D = x->shape[x->ndim - 1];
  LC_CHECK(D % 2 == 0, "rope: head dim must be even");
  int odt = is_float(x->dtype) ? x->dtype : LC_F32;
  LcTensor* y = alloc(odt, x->dims());
  int64_t rows = L ? x->numel() / D : 0;
  if (rows && D) {
    int cap = 0;
    const float* cs = rope_table((int)D, base, (int)L, &cap);
    TV v = tv(x);
    if (x->dtype != odt) {  // integer input: convert first
      LcTensor* f = alloc(odt, x->dims());
      copy_into(x, f);
      v = tv(f);
      k_rope<<<blocks_for(rows * (D / 2), 256), 256, 0, stream()>>>(v, cs, rows, L, (int)(D / 2), cap, y->data());
      release(f);
    } else if ((D / 2) % 4 == 0 && x->strides[x->ndim - 1] == 1 && rows < INT32_MAX && L < INT32_MAX && x->ndim <= 5 &&
               (odt == LC_F32 || odt == LC_F16 || odt == LC_BF16) && ((uintptr_t)x->data() % (4 * dtype_size(odt))) == 0 &&
               [&] {
                 for (int d = 0; d < x->ndim - 1; d++)
                   if ((x->shape[d] > 1 && x->strides[d] % 4) || x->shape[d] >= INT32_MAX) return false;  // a size-1 axis's stride is never used
                 return true;
               }()) {
      const bool v8 = odt != LC_F32 && (D / 2) % 8 == 0 && ((uintptr_t)x->data() % 16) == 0 && [&] {
        for (int d = 0; d < x->ndim - 1; d++)
          if (x->shape[d] > 1 && x->strides[d] % 8) return false;
        return true;
      }();
      const unsigned blocks = blocks_for(rows * (D / (v8 ? 16 : 8)), 256);
      if (v8 && odt == LC_F16)
        lc::launch_chain(k_rope_vec8<__half>, dim3(blocks), dim3(256), 0, stream(), v, cs, (int)rows, (int)L, (int)(D / 2), cap, (__half*)y->data());
      else if (v8)
        lc::launch_chain(k_rope_vec8<__nv_bfloat16>, dim3(blocks), dim3(256), 0, stream(), v, cs, (int)rows, (int)L, (int)(D / 2), cap,
                         (__nv_bfloat16*)y->data());
      else if (odt == LC_F32) lc::launch_chain(k_rope_vec<float>, dim3(blocks), dim3(256), 0, stream(), v, cs, (int)rows, (int)L, (int)(D / 2), cap, (float*)y->data());
      else if (odt == LC_F16) lc::launch_chain(k_rope_vec<__half>, dim3(blocks), dim3(256), 0, stream(), v, cs, (int)rows, (int)L, (int)(D / 2), cap, (__half*)y->data());
      else lc::launch_chain(k_rope_vec<__nv_bfloat16>, dim3(blocks), dim3(256), 0, stream(), v, cs, (int)rows, (int)L, (int)(D / 2), cap, (__nv_bfloat16*)y->data());
    } else {
      k_rope<<<blocks_for(rows * (D / 2), 256), 256, 0, stream()>>>(v, cs, rows, L, (int)(D / 2), cap, y->data());
    }
    LC_LAUNCHED(1);
  }
  *out = handle(y);
  LC_API_END
}

int lc_sdpa(lc_tensor* out, lc_tensor qh, lc_tensor kh, lc_tensor vh, lc_tensor mh, double scale) {
  LC_API_BEGIN
  LcTensor* q = check(qh, "sdpa q");
  LcTensor* k = check(kh, "sdpa k");
  LcTensor* v = check(vh, "sdpa v");
  LcTensor* m = mh ? check(mh, "sdpa mask") : nullptr;
  LC_CHECK(q->ndim == 4 && k->ndim == 4 && v->ndim == 4, "sdpa: q/k/v must be [B, H, L, D]");
  int64_t B = q->shape[0], H = q->shape[1], Lq = q->shape[2], D = q->shape[3];
  int64_t Lk = k->shape[2], Dv = v->shape[3];
  LC_CHECK(k->shape[0] == B && v->shape[0] == B && k->shape[1] == H && v->shape[1] == H, "sdpa: batch/head mismatch");
  LC_CHECK(k->shape[3] == D && v->shape[2] == Lk, "sdpa: k/v shapes do not match q");
  if (m) LC_CHECK(m->dtype == LC_BOOL, "sdpa: the mask must be bool (additive float masks are not part of the contract)");
  int odt = is_float(q->dtype) ? q->dtype : LC_F32;
  LcTensor* y = alloc(odt, {B, H, Lq, Dv});
  if (B * H * Lq && Dv) {
    TV mv{};
    if (m) mv = tv_broadcast(m, {B, H, Lq, Lk});
    LcTensor* ytc = nullptr;
    if (odt == q->dtype && lc::sdpa_tc(q, k, v, m, (float)scale, &ytc)) {  // f16/bf16, head dim 64: tcgen05
      release(y);
      *out = handle(ytc);
      return 0;
    }
    if (lc::sdpa_flash(q, k, v, m, (float)scale, y)) {
      *out = handle(y);
      return 0;
    }
    LC_CHECK(D <= SDPA_MAXD && Dv <= SDPA_MAXD, "sdpa: head dim above 256 is not supported");
    unsigned blocks = (unsigned)((B * H * Lq + 3) / 4);
    k_sdpa_generic<<<blocks, 128, 0, stream()>>>(tv(q), tv(k), tv(v), mv, m ? 1 : 0, (float)scale, y->data(), odt, B, H, Lq, Lk,
                                                (int)D, (int)Dv);
    LC_LAUNCHED(1);
  }
  *out = handle(y);
  LC_API_END
}

int lc_geglu(lc_tensor* out, lc_tensor xh) {
  LC_API_BEGIN
  LcTensor* x0 = check(xh, "geglu");
  LC_CHECK(x0->ndim >= 1 && x0->shape[x0->ndim - 1] % 2 == 0, "geglu: last axis must be even");
  int64_t F = x0->shape[x0->ndim - 1] / 2;
  std::vector<int64_t> sh = x0->dims();
  sh.back() = F;
  int odt = is_float(x0->dtype) ? x0->dtype : LC_F32;
  LcTensor* y = alloc(odt, sh);
  int64_t rows = F ? y->numel() / F : 0;
  if (rows) {
    LcTensor* x = contiguous(x0);
    int vn = x->dtype == LC_F32 ? 4 : 8;
    bool vec = x->dtype == odt && (odt == LC_F32 || is_half(odt)) && F % vn == 0 &&
               ((((uintptr_t)x->data()) | ((uintptr_t)y->data())) & 15) == 0;
    cudaStream_t st = stream();
    if (vec) {
      unsigned blocks = blocks_for(rows * F / vn, 256);
      if (odt == LC_F16) lc::launch_chain(k_geglu_vec<__half>, dim3(blocks), dim3(256), 0, st, (const __half*)x->data(), (__half*)y->data(), rows, F);
      else if (odt == LC_BF16) lc::launch_chain(k_geglu_vec<__nv_bfloat16>, dim3(blocks), dim3(256), 0, st, (const __nv_bfloat16*)x->data(), (__nv_bfloat16*)y->data(), rows, F);
      else lc::launch_chain(k_geglu_vec<float>, dim3(blocks), dim3(256), 0, st, (const float*)x->data(), (float*)y->data(), rows, F);
    } else if (x->dtype == LC_F64) {
      k_geglu_generic<double><<<blocks_for(rows * F, 256), 256, 0, st>>>(x->data(), x->dtype, y->data(), odt, rows, F);
    } else {
      k_geglu_generic<float><<<blocks_for(rows * F, 256), 256, 0, st>>>(x->data(), x->dtype, y->data(), odt, rows, F);
    }
    LC_LAUNCHED(1);
    if (x != x0) release(x);
  }
  *out = handle(y);
  LC_API_END
}

int lc_mean_pool(lc_tensor* out, lc_tensor xh, lc_tensor mh) {
  LC_API_BEGIN
  LcTensor* x0 = check(xh, "meanPool x");
  LcTensor* m0 = check(mh, "meanPool mask");
  LC_CHECK(x0->ndim == 3 && m0->ndim == 2 && m0->shape[0] == x0->shape[0] && m0->shape[1] == x0->shape[1],
           "meanPool: x [B, L, D] and mask [B, L] expected");
  int64_t B = x0->shape[0], L = x0->shape[1], D = x0->shape[2];
  LcTensor* y = alloc(LC_F32, {B, D});
  if (B * D) {
    LcTensor* x = contiguous(x0);
    LcTensor* m = contiguous(m0);
    const int d = x->dtype;
    const int vec = d == LC_F32 ? 4 : 8;
    const int64_t LS = (L + 255) / 256;
    if ((d == LC_F16 || d == LC_BF16 || d == LC_F32) && D % vec == 0 && B <= 65535 && LS <= 65535) {
      dim3 grid((unsigned)((D + 32 * vec - 1) / (32 * vec)), (unsigned)B, (unsigned)std::max<int64_t>(LS, 1));
      float* part = LS > 1 ? (float*)dmalloc((size_t)(LS * B * D + LS * B) * sizeof(float)) : nullptr;
      float* pcnt = part ? part + LS * B * D : nullptr;
      if (d == LC_F16)
        lc::launch_chain(k_mean_pool_vec<__half>, grid, dim3(256), 0, stream(), (const __half*)x->data(), (const char*)m->data(), (int)m->dtype,
                         (float*)y->data(), part, pcnt, L, D);
      else if (d == LC_BF16)
        lc::launch_chain(k_mean_pool_vec<__nv_bfloat16>, grid, dim3(256), 0, stream(), (const __nv_bfloat16*)x->data(), (const char*)m->data(),
                         (int)m->dtype, (float*)y->data(), part, pcnt, L, D);
      else
        lc::launch_chain(k_mean_pool_vec<float>, grid, dim3(256), 0, stream(), (const float*)x->data(), (const char*)m->data(), (int)m->dtype,
                         (float*)y->data(), part, pcnt, L, D);
      if (part) {
        LC_LAUNCHED(1);
        lc::launch_chain(k_mean_pool_fin, dim3(blocks_for(B * D, 256)), dim3(256), 0, stream(), (const float*)part, (const float*)pcnt,
                         (float*)y->data(), B, D, (int)LS);
        dfree(part);
      }
    } else {
      k_mean_pool<<<blocks_for(B * D, 256), 256, 0, stream()>>>(x->data(), x->dtype, m->data(), m->dtype, (float*)y->data(), B, L, D);
    }
    LC_LAUNCHED(1);
    if (x != x0) release(x);
    if (m != m0) release(m);
  }
  *out = handle(y);
  LC_API_END
}

int lc_matmul(lc_tensor* out, lc_tensor ah, lc_tensor bh) {
  LC_API_BEGIN
  LcTensor* a0 = check(ah, "matmul a");
  LcTensor* b0 = check(bh, "matmul b");
  LC_CHECK(a0->ndim >= 2 && b0->ndim >= 2, "matmul: operands must be at least 2-D");
  int64_t m = a0->shape[a0->ndim - 2], k = a0->shape[a0->ndim - 1];
  int64_t k2 = b0->shape[b0->ndim - 2], n = b0->shape[b0->ndim - 1];
  LC_CHECK(k == k2, "matmul: inner dimensions differ");
  std::vector<int64_t> ba(a0->shape, a0->shape + a0->ndim - 2), bb(b0->shape, b0->shape + b0->ndim - 2);
  std::vector<int64_t> bs = broadcast_shapes({ba, bb});
  LC_CHECK(bs.size() <= 6, "matmul: at most 6 batch dims");
  std::vector<int64_t> osh = bs;
  osh.push_back(m);
  osh.push_back(n);
  int odt = float_out(a0->dtype, b0->dtype);
  LcTensor* y = alloc(odt, osh);
  int64_t batch = 1;
  for (auto d : bs) batch *= d;
  if (batch && m && n) {
    MM p{};
    p.a = a0->data(); p.adt = a0->dtype;
    p.b = b0->data(); p.bdt = b0->dtype;
    p.c = y->data(); p.cdt = odt;
    p.m = m; p.n = n; p.k = k;
    p.sam = a0->strides[a0->ndim - 2]; p.sak = a0->strides[a0->ndim - 1];
    p.sbk = b0->strides[b0->ndim - 2]; p.sbn = b0->strides[b0->ndim - 1];
    p.nb = (int)bs.size();
    for (int i = 0; i < p.nb; i++) {
      p.bshape[i] = bs[i];
      int ia = i - (p.nb - (a0->ndim - 2)), ib = i - (p.nb - (b0->ndim - 2));
      p.bsa[i] = (ia >= 0 && a0->shape[ia] != 1) ? a0->strides[ia] : 0;
      p.bsb[i] = (ib >= 0 && b0->shape[ib] != 1) ? b0->strides[ib] : 0;
    }
    // data() already includes the view offset
    launch_mm(p, batch, odt == LC_F64);
  }
  *out = handle(y);
  LC_API_END
}

int lc_linear(lc_tensor* out, lc_tensor xh, lc_tensor wh, lc_tensor bh) {
  LC_API_BEGIN
  LcTensor* x0 = check(xh, "linear x");
  LcTensor* w0 = check(wh, "linear w");
  LcTensor* b0 = bh ? check(bh, "linear bias") : nullptr;
  LC_CHECK(x0->ndim >= 1 && w0->ndim == 2, "linear: x [..., in] and w [out, in] expected");
  int64_t K = x0->shape[x0->ndim - 1], N = w0->shape[0];
  LC_CHECK(w0->shape[1] == K, "linear: x [" + std::to_string(K) + "] vs w " + shape_str(w0->dims()));
  if (b0) LC_CHECK(b0->numel() == N, "linear: bias size differs from out features");
  std::vector<int64_t> sh = x0->dims();
  sh.back() = N;
  int odt = is_float(x0->dtype) ? x0->dtype : LC_F32;
  LcTensor* y = alloc(odt, sh);
  int64_t M = K ? x0->numel() / K : 0;
  if (M && N) {
    LcTensor* x = contiguous(x0);
    LcTensor* w = contiguous(w0);
    LcTensor* b = b0 ? contiguous(b0) : nullptr;
    LcTensor* x2 = view_of(x, {M, K}, {K, 1}, x->offset);
    bool done = false;
    // Few rows of a small product (a head over a handful of marker rows, a
    // one-row projection): a warp per output finishes before the tensor-core
    // GEMM's pipeline fills.
    const bool few = M <= 16 && M * N * K <= ((int64_t)1 << 23);
    if (!few && is_half(odt) && x->dtype == odt && w->dtype == odt && (!b || is_float(b->dtype))) {
      GemmEpilogue ep{};
      ep.w_static = w == w0 && upload_settled(w->st);  // weight blocks requested before the dependency wait
      done = gemm_linear(x2, w, b, y, ep);
    }
    if (!done) {
      LcTensor* y2 = view_of(y, {M, N}, {N, 1}, 0);
      linear_simt(x2, w, b, y2);
      release(y2);
    }
    release(x2);
    if (x != x0) release(x);
    if (w != w0) release(w);
    if (b && b != b0) release(b);
  } else if (M && N == 0) {
  } else if (N) {
    // K == 0: y = bias (or zeros)
    CUDA_OK(cudaMemsetAsync(y->data(), 0, y->numel() * dtype_size(odt), stream()));
  }
  *out = handle(y);
  LC_API_END
}

}  // extern "C"
