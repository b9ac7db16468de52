// Axis reductions, softmax, scans and sort
// (packages/tensor-backend/src/index.ts:200-206 and 300-315).
//
// The input is viewed as [outer, n, inner] around the reduced axis. When
// inner == 1 one warp reduces one row with shuffles; otherwise one thread
// walks one (outer, inner) column, which keeps loads coalesced across the
// threads of a warp.
#include "lc_api.h"

#include <cfloat>
#include <climits>

enum RedOp : int { R_SUM, R_MAX, R_MIN, R_MEAN, R_ARGMAX, R_ARGMIN };

template <typename CT> __device__ __forceinline__ bool is_nan_v(CT) { return false; }
template <> __device__ __forceinline__ bool is_nan_v<float>(float v) { return isnan(v); }
template <> __device__ __forceinline__ bool is_nan_v<double>(double v) { return isnan(v); }

// a "beats" b for max (NaN propagates, ties keep the earlier index)
template <typename CT>
__device__ __forceinline__ bool better(int op, CT a, int64_t ia, CT b, int64_t ib) {
  bool na = is_nan_v(a), nb = is_nan_v(b);
  if (na || nb) return na && (!nb || ia < ib);
  bool mx = (op == R_MAX || op == R_ARGMAX);
  if (a == b) return ia < ib;
  return mx ? (a > b) : (a < b);
}

template <typename CT, typename AT>
__device__ void reduce_store(int op, char* out, int out_dtype, int64_t oi, AT acc, CT best, int64_t bi, int64_t n) {
  switch (op) {
    case R_SUM: st_as<AT>(out, out_dtype, oi, acc); break;
    case R_MEAN: st_as<double>(out, out_dtype, oi, (double)acc / (double)n); break;
    case R_MAX: case R_MIN: st_as<CT>(out, out_dtype, oi, best); break;
    default: st_as<int64_t>(out, out_dtype, oi, bi); break;
  }
}

// one warp per row (inner == 1)
template <typename CT, typename AT>
__global__ void k_reduce_rows(const char* x, int dtype, char* out, int out_dtype, int op, int64_t rows, int64_t n) {
  int lane = threadIdx.x & 31;
  int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += nwarps) {
    AT acc = 0;
    CT best = 0;
    int64_t bi = -1;
    for (int64_t j = lane; j < n; j += 32) {
      CT v = ld_as<CT>(x, dtype, r * n + j);
      if (op == R_SUM || op == R_MEAN) acc += (AT)v;
      else if (bi < 0 || better<CT>(op, v, j, best, bi)) { best = v; bi = j; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      AT a2 = __shfl_xor_sync(0xffffffffu, acc, o);
      CT b2 = __shfl_xor_sync(0xffffffffu, best, o);
      int64_t i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      if (op == R_SUM || op == R_MEAN) acc += a2;
      else if (i2 >= 0 && (bi < 0 || better<CT>(op, b2, i2, best, bi))) { best = b2; bi = i2; }
    }
    if (lane == 0) reduce_store<CT, AT>(op, out, out_dtype, r, acc, best, bi, n);
  }
}

// one thread per (outer, inner) column
template <typename CT, typename AT>
__global__ void k_reduce_cols(const char* x, int dtype, char* out, int out_dtype, int op, int64_t outer, int64_t n, int64_t inner) {
  LC_GRID_STRIDE(c, outer * inner) {
    int64_t o = c / inner, i = c % inner;
    int64_t base = o * n * inner + i;
    AT acc = 0;
    CT best = 0;
    int64_t bi = -1;
    for (int64_t j = 0; j < n; j++) {
      CT v = ld_as<CT>(x, dtype, base + j * inner);
      if (op == R_SUM || op == R_MEAN) acc += (AT)v;
      else if (bi < 0 || better<CT>(op, v, j, best, bi)) { best = v; bi = j; }
    }
    reduce_store<CT, AT>(op, out, out_dtype, c, acc, best, bi, n);
  }
}

// softmax: f32 math (f64 for f64)
template <typename CT>
__global__ void k_softmax_rows(const char* x, int dtype, char* out, int out_dtype, int64_t rows, int64_t n) {
  int lane = threadIdx.x & 31;
  int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += nwarps) {
    CT m = -INFINITY;
    for (int64_t j = lane; j < n; j += 32) m = fmax(m, ld_as<CT>(x, dtype, r * n + j));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
    CT s = 0;
    for (int64_t j = lane; j < n; j += 32) s += exp(ld_as<CT>(x, dtype, r * n + j) - m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    CT inv = (CT)1 / s;
    for (int64_t j = lane; j < n; j += 32) st_as<CT>(out, out_dtype, r * n + j, exp(ld_as<CT>(x, dtype, r * n + j) - m) * inv);
  }
}

template <typename CT>
__global__ void k_softmax_cols(const char* x, int dtype, char* out, int out_dtype, int64_t outer, int64_t n, int64_t inner) {
  LC_GRID_STRIDE(c, outer * inner) {
    int64_t o = c / inner, i = c % inner;
    int64_t base = o * n * inner + i;
    CT m = -INFINITY;
    for (int64_t j = 0; j < n; j++) m = fmax(m, ld_as<CT>(x, dtype, base + j * inner));
    CT s = 0;
    for (int64_t j = 0; j < n; j++) s += exp(ld_as<CT>(x, dtype, base + j * inner) - m);
    CT inv = (CT)1 / s;
    for (int64_t j = 0; j < n; j++) st_as<CT>(out, out_dtype, base + j * inner, exp(ld_as<CT>(x, dtype, base + j * inner) - m) * inv);
  }
}

// ---- dense 16-bit / f32 rows, one warp per row held in registers
// (16-byte loads, each element read once): the fast paths of softmax and of
// sum / mean / max / min over the last axis. n % (16 / sizeof(T)) == 0 and
// n <= 32 * (16 / sizeof(T)) * MAXV.
template <typename T, int MAXV>
__global__ void __launch_bounds__(256) k_softmax_rows_vec(const T* __restrict__ x, T* __restrict__ y, int64_t rows, int n) {
  pdl_trigger();
  pdl_wait();
  constexpr int VEC = 16 / sizeof(T);
  // short rows (up to 4 vectors per lane) keep the values and then the
  // exponentials as floats; longer rows stay in registers in their stored
  // form (4 registers per 16-byte vector), each pass converts what it reads
  // and the exponentials are recomputed for the output (same values, same order)
  constexpr bool KEEP_F = MAXV <= 4;
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int nv = n / VEC;
  // 16-bit outputs: the hardware exp2 (relative error ~2^-22, far below the
  // output's 2^-11 rounding); f32 outputs keep the full expf
  auto ex = [](float v) { if constexpr (sizeof(T) == 2) return __expf(v); else return expf(v); };
  for (int64_t r = warp; r < rows; r += nwarps) {
    uint4 raw[KEEP_F ? 1 : MAXV];
    float v[KEEP_F ? MAXV : 1][VEC];
    float m = -INFINITY;
#pragma unroll
    for (int t = 0; t < MAXV; t++) {
      const int c = t * 32 + lane;
      if (c < nv) {
        const uint4 ld = *(const uint4*)(x + r * n + (int64_t)c * VEC);
        const T* e = (const T*)&ld;
        if constexpr (!KEEP_F) raw[t] = ld;
#pragma unroll
        for (int j = 0; j < VEC; j++) {
          const float f = to_f<T>(e[j]);
          if constexpr (KEEP_F) v[t][j] = f;
          m = fmaxf(m, f);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
#pragma unroll
    for (int t = 0; t < MAXV; t++)
      if (t * 32 + lane < nv) {
#pragma unroll
        for (int j = 0; j < VEC; j++) {
          if constexpr (KEEP_F) {
            v[t][j] = ex(v[t][j] - m);
            s += v[t][j];
          } else {
            s += ex(to_f<T>(((const T*)&raw[t])[j]) - m);
          }
        }
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float inv = 1.f / s;
#pragma unroll
    for (int t = 0; t < MAXV; t++) {
      const int c = t * 32 + lane;
      if (c < nv) {
        uint4 o4;
        T* q = (T*)&o4;
#pragma unroll
        for (int j = 0; j < VEC; j++) {
          if constexpr (KEEP_F) q[j] = from_f<T>(v[t][j] * inv);
          else q[j] = from_f<T>(ex(to_f<T>(((const T*)&raw[t])[j]) - m) * inv);
        }
        *(uint4*)(y + r * n + (int64_t)c * VEC) = o4;
      }
    }
  }
}

// max / min with NaN propagation (the generic path's rule)
__device__ __forceinline__ float pick(int op, float a, float b) {
  if (isnan(a) || isnan(b)) return isnan(a) ? a : b;
  return op == R_MAX ? fmaxf(a, b) : fminf(a, b);
}

// max / min of the values of one 16-byte vector folded into a running value:
// 16-bit types as packed pairs with NaN propagation (__hmax2_nan / __hmin2_nan,
// exact), f32 with fmaxf / fminf and a NaN flag, so no per-element NaN branch
template <typename T> struct Pair2;
template <> struct Pair2<__half> { using type = __half2; };
template <> struct Pair2<__nv_bfloat16> { using type = __nv_bfloat162; };
template <typename T, int OP>
struct VecPick {
  using P = typename Pair2<T>::type;
  P acc;
  __device__ __forceinline__ VecPick() {
    const T init = from_f<T>(OP == R_MAX ? -INFINITY : INFINITY);
    acc = P(init, init);
  }
  __device__ __forceinline__ void add(const uint4& raw) {
    const P* p = (const P*)&raw;
#pragma unroll
    for (int k = 0; k < 4; k++) acc = OP == R_MAX ? __hmax2_nan(acc, p[k]) : __hmin2_nan(acc, p[k]);
  }
  __device__ __forceinline__ float value() const { return pick(OP, to_f<T>(acc.x), to_f<T>(acc.y)); }
};
template <int OP>
struct VecPick<float, OP> {
  float acc = OP == R_MAX ? -INFINITY : INFINITY;
  bool nan = false;
  __device__ __forceinline__ void add(const uint4& raw) {
    const float* f = (const float*)&raw;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      acc = OP == R_MAX ? fmaxf(acc, f[k]) : fminf(acc, f[k]);
      nan |= f[k] != f[k];
    }
  }
  __device__ __forceinline__ float value() const { return nan ? __int_as_float(0x7fc00000) : acc; }
};

// sum (f32 accumulation), mean (f64), max, min over each row; the operation
// is a template parameter so the per-element loop carries no branch on it
template <typename T, int MAXV, int OP>
__global__ void __launch_bounds__(256) k_reduce_rows_vec(const T* __restrict__ x, char* out, int out_dtype, int64_t rows, int n) {
  pdl_trigger();
  pdl_wait();
  constexpr int VEC = 16 / sizeof(T);
  constexpr int op = OP;
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int nv = n / VEC;
  constexpr bool mm = op == R_MAX || op == R_MIN;
  for (int64_t r = warp; r < rows; r += nwarps) {
    float acc = 0.f, best = op == R_MAX ? -INFINITY : INFINITY;
    double dacc = 0.0;
    VecPick<T, mm ? op : R_MAX> vp;
#pragma unroll
    for (int t = 0; t < MAXV; t++) {
      const int c = t * 32 + lane;
      if (c < nv) {
        const uint4 raw = *(const uint4*)(x + r * n + (int64_t)c * VEC);
        if constexpr (mm) {
          vp.add(raw);
        } else {
          const T* e = (const T*)&raw;
#pragma unroll
          for (int j = 0; j < VEC; j++) {
            const float f = to_f<T>(e[j]);
            if constexpr (op == R_MEAN) dacc += (double)f;
            else acc += f;
          }
        }
      }
    }
    if constexpr (mm) best = vp.value();
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      if constexpr (mm) best = pick(op, best, __shfl_xor_sync(0xffffffffu, best, o));
      else if constexpr (op == R_MEAN) dacc += __shfl_xor_sync(0xffffffffu, dacc, o);
      else acc += __shfl_xor_sync(0xffffffffu, acc, o);
    }
    if (lane == 0) {
      if constexpr (mm) st_as<float>(out, out_dtype, r, best);
      else if constexpr (op == R_MEAN) st_as<double>(out, out_dtype, r, dacc / (double)n);
      else st_as<float>(out, out_dtype, r, acc);
    }
  }
}

// ---- rows longer than one warp's register tile: one 256-thread block per row
// (rows taken in turn by the grid), each thread holding up to MAXV 16-byte
// vectors; warp shuffles, then the 8 warps' partials through shared memory,
// read by every thread in the same order.
template <typename A>
__device__ __forceinline__ A block_sum256(A v, A* sm) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = v;
  __syncthreads();
  A t = sm[0];
#pragma unroll
  for (int w = 1; w < 8; w++) t += sm[w];
  __syncthreads();
  return t;
}
template <int OP>
__device__ __forceinline__ float block_pick256(float v, float* sm) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = pick(OP, v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = sm[0];
#pragma unroll
  for (int w = 1; w < 8; w++) t = pick(OP, t, sm[w]);
  __syncthreads();
  return t;
}

template <typename T, int MAXV>
__global__ void __launch_bounds__(256) k_softmax_rows_blk(const T* __restrict__ x, T* __restrict__ y, int64_t rows, int n) {
  constexpr int VEC = 16 / sizeof(T);
  __shared__ float sm[8];
  const int nv = n / VEC;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    float v[MAXV][VEC];
    float m = -INFINITY;
#pragma unroll
    for (int t = 0; t < MAXV; t++) {
      const int c = t * 256 + threadIdx.x;
      if (c < nv) {
        const uint4 raw = *(const uint4*)(x + r * n + (int64_t)c * VEC);
        const T* e = (const T*)&raw;
#pragma unroll
        for (int j = 0; j < VEC; j++) {
          v[t][j] = to_f<T>(e[j]);
          m = fmaxf(m, v[t][j]);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = m;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < 8; w++) m = fmaxf(m, sm[w]);
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int t = 0; t < MAXV; t++)
      if (t * 256 + (int)threadIdx.x < nv)
#pragma unroll
        for (int j = 0; j < VEC; j++) {
          if constexpr (sizeof(T) == 2) v[t][j] = __expf(v[t][j] - m);
          else v[t][j] = expf(v[t][j] - m);
          s += v[t][j];
        }
    s = block_sum256<float>(s, sm);
    const float inv = 1.f / s;
#pragma unroll
    for (int t = 0; t < MAXV; t++) {
      const int c = t * 256 + threadIdx.x;
      if (c < nv) {
        uint4 raw;
        T* e = (T*)&raw;
#pragma unroll
        for (int j = 0; j < VEC; j++) e[j] = from_f<T>(v[t][j] * inv);
        *(uint4*)(y + r * n + (int64_t)c * VEC) = raw;
      }
    }
  }
}

template <typename T, int MAXV, int OP>
__global__ void __launch_bounds__(256) k_reduce_rows_blk(const T* __restrict__ x, char* out, int out_dtype, int64_t rows, int n) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr bool mm = OP == R_MAX || OP == R_MIN;
  __shared__ double smd[8];
  __shared__ float smf[8];
  const int nv = n / VEC;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    float acc = 0.f, best = OP == R_MAX ? -INFINITY : INFINITY;
    double dacc = 0.0;
    VecPick<T, mm ? OP : R_MAX> vp;
#pragma unroll
    for (int t = 0; t < MAXV; t++) {
      const int c = t * 256 + threadIdx.x;
      if (c < nv) {
        const uint4 raw = *(const uint4*)(x + r * n + (int64_t)c * VEC);
        if constexpr (mm) {
          vp.add(raw);
        } else {
          const T* e = (const T*)&raw;
#pragma unroll
          for (int j = 0; j < VEC; j++) {
            const float f = to_f<T>(e[j]);
            if constexpr (OP == R_MEAN) dacc += (double)f;
            else acc += f;
          }
        }
      }
    }
    if constexpr (mm) best = vp.value();
    if constexpr (mm) best = block_pick256<OP>(best, smf);
    else if constexpr (OP == R_MEAN) dacc = block_sum256<double>(dacc, smd);
    else acc = block_sum256<float>(acc, smf);
    if (threadIdx.x == 0) {
      if constexpr (mm) st_as<float>(out, out_dtype, r, best);
      else if constexpr (OP == R_MEAN) st_as<double>(out, out_dtype, r, dacc / (double)n);
      else st_as<float>(out, out_dtype, r, acc);
    }
  }
}

// inclusive prefix sum, one thread per column, wrapping in the output dtype
template <typename CT>
__global__ void k_cumsum(const char* x, int dtype, char* out, int out_dtype, int64_t outer, int64_t n, int64_t inner) {
  LC_GRID_STRIDE(c, outer * inner) {
    int64_t o = c / inner, i = c % inner;
    int64_t base = o * n * inner + i;
    CT acc = 0;
    for (int64_t j = 0; j < n; j++) {
      acc += ld_as<CT>(x, dtype, base + j * inner);
      if (out_dtype != LC_F32 && out_dtype != LC_F64 && out_dtype != LC_F16 && out_dtype != LC_BF16 && out_dtype != LC_U64 && out_dtype != LC_I64) {
        // wrap to the output width so later sums continue from the wrapped value
        st_as<CT>(out, out_dtype, base + j * inner, acc);
        acc = ld_as<CT>(out, out_dtype, base + j * inner);
      } else {
        st_as<CT>(out, out_dtype, base + j * inner, acc);
        if (out_dtype == LC_F16 || out_dtype == LC_BF16) acc = ld_as<CT>(out, out_dtype, base + j * inner);
      }
    }
  }
}

// ascending bitonic sort of one row per block in shared memory (NaN last)
template <typename CT> __device__ __forceinline__ CT sort_pad();
template <> __device__ __forceinline__ float sort_pad<float>() { return __int_as_float(0x7fc00000); }
template <> __device__ __forceinline__ double sort_pad<double>() { return __longlong_as_double(0x7ff8000000000000ll); }
template <> __device__ __forceinline__ int64_t sort_pad<int64_t>() { return LLONG_MAX; }
template <> __device__ __forceinline__ uint64_t sort_pad<uint64_t>() { return ULLONG_MAX; }

template <typename CT>
__device__ __forceinline__ bool sort_lt(CT a, CT b) {
  bool na = is_nan_v(a), nb = is_nan_v(b);
  if (na || nb) return !na && nb;
  return a < b;
}

template <typename CT>
__global__ void k_sort_rows(const char* x, int dtype, char* out, int64_t n, int P) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  CT* s = (CT*)smem_raw;
  int64_t r = blockIdx.x;
  for (int i = threadIdx.x; i < P; i += blockDim.x) s[i] = i < n ? ld_as<CT>(x, dtype, r * n + i) : sort_pad<CT>();
  __syncthreads();
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        int p = i ^ j;
        if (p > i) {
          bool up = (i & k) == 0;
          CT a = s[i], b = s[p];
          if (up ? sort_lt(b, a) : sort_lt(a, b)) {
            s[i] = b;
            s[p] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) st_as<CT>(out, dtype, r * n + i, s[i]);
}

using namespace lc;

namespace {

struct Axis3 {
  int64_t outer, n, inner;
};
Axis3 split_axis(const LcTensor* x, int a) {
  Axis3 s{1, x->shape[a], 1};
  for (int i = 0; i < a; i++) s.outer *= x->shape[i];
  for (int i = a + 1; i < x->ndim; i++) s.inner *= x->shape[i];
  return s;
}

std::vector<int64_t> reduced_shape(const LcTensor* x, int a, bool keep) {
  std::vector<int64_t> sh;
  for (int i = 0; i < x->ndim; i++) {
    if (i == a) {
      if (keep) sh.push_back(1);
    } else sh.push_back(x->shape[i]);
  }
  return sh;
}

// Fast-path dispatch: dense f16 / bf16 / f32 rows of at most 32 * VEC * 8
// elements, n a multiple of the vector width. Returns false when it does not apply.
// `maxv` vectors per lane at most (softmax keeps them in registers: 12; the
// reductions only stream them: 24).
bool row_vec_ok(int dtype, int64_t n, int64_t rows, int maxv) {
  if (!(dtype == LC_F16 || dtype == LC_BF16 || dtype == LC_F32) || rows <= 0) return false;
  const int vec = dtype == LC_F32 ? 4 : 8;
  return n > 0 && n % vec == 0 && n <= (int64_t)32 * vec * maxv && n < INT32_MAX;
}
// Block-per-row path: dense f16 / bf16 / f32 rows longer than the warp path
// takes, up to 256 threads x 8 vectors, 16-byte aligned.
bool row_blk_ok(int dtype, int64_t n, int64_t rows, const void* p) {
  if (!(dtype == LC_F16 || dtype == LC_BF16 || dtype == LC_F32) || rows <= 0 || ((uintptr_t)p & 15)) return false;
  const int vec = dtype == LC_F32 ? 4 : 8;
  return n > 0 && n % vec == 0 && n <= 256 * vec * 8 && n < INT32_MAX;
}
int row_blk_maxv(int dtype, int64_t n) {
  const int vec = dtype == LC_F32 ? 4 : 8;
  const int per = (int)((n / vec + 255) / 256);
  return per <= 1 ? 1 : per <= 2 ? 2 : per <= 4 ? 4 : 8;
}
unsigned row_blk_grid(int64_t rows) { return (unsigned)std::min<int64_t>(rows, (int64_t)num_sms() * 8); }
int row_vec_maxv(int dtype, int64_t n) {
  const int vec = dtype == LC_F32 ? 4 : 8;
  const int per = (int)((n / vec + 31) / 32);
  return per <= 1 ? 1 : per <= 2 ? 2 : per <= 4 ? 4 : per <= 8 ? 8 : per <= 12 ? 12 : per <= 16 ? 16 : 24;
}

#define LC_ROWVEC_DISPATCH(KERNEL, T, MAXV_RT, BLOCKS, ...)                     \
  switch (MAXV_RT) {                                                           \
    case 1: KERNEL<T, 1><<<BLOCKS, 256, 0, stream()>>>(__VA_ARGS__); break;    \
    case 2: KERNEL<T, 2><<<BLOCKS, 256, 0, stream()>>>(__VA_ARGS__); break;    \
    case 4: KERNEL<T, 4><<<BLOCKS, 256, 0, stream()>>>(__VA_ARGS__); break;    \
    default: KERNEL<T, 8><<<BLOCKS, 256, 0, stream()>>>(__VA_ARGS__); break;   \
  }

template <typename T, int MAXV>
void launch_reduce_vec_op(unsigned blocks, int op, const T* x, char* out, int odt, int64_t rows, int n) {
  switch (op) {
    case R_SUM: lc::launch_chain(k_reduce_rows_vec<T, MAXV, R_SUM>, dim3(blocks), dim3(256), 0, stream(), x, out, odt, rows, n); break;
    case R_MEAN: lc::launch_chain(k_reduce_rows_vec<T, MAXV, R_MEAN>, dim3(blocks), dim3(256), 0, stream(), x, out, odt, rows, n); break;
    case R_MAX: lc::launch_chain(k_reduce_rows_vec<T, MAXV, R_MAX>, dim3(blocks), dim3(256), 0, stream(), x, out, odt, rows, n); break;
    default: lc::launch_chain(k_reduce_rows_vec<T, MAXV, R_MIN>, dim3(blocks), dim3(256), 0, stream(), x, out, odt, rows, n); break;
  }
}
template <typename T, int MAXV>
void launch_reduce_blk_op(unsigned blocks, int op, const T* x, char* out, int odt, int64_t rows, int n) {
  switch (op) {
    case R_SUM: k_reduce_rows_blk<T, MAXV, R_SUM><<<blocks, 256, 0, stream()>>>(x, out, odt, rows, n); break;
    case R_MEAN: k_reduce_rows_blk<T, MAXV, R_MEAN><<<blocks, 256, 0, stream()>>>(x, out, odt, rows, n); break;
    case R_MAX: k_reduce_rows_blk<T, MAXV, R_MAX><<<blocks, 256, 0, stream()>>>(x, out, odt, rows, n); break;
    default: k_reduce_rows_blk<T, MAXV, R_MIN><<<blocks, 256, 0, stream()>>>(x, out, odt, rows, n); break;
  }
}
template <typename T>
void launch_reduce_blk(unsigned blocks, int maxv, int op, const T* x, char* out, int odt, int64_t rows, int n) {
  switch (maxv) {
    case 1: launch_reduce_blk_op<T, 1>(blocks, op, x, out, odt, rows, n); break;
    case 2: launch_reduce_blk_op<T, 2>(blocks, op, x, out, odt, rows, n); break;
    case 4: launch_reduce_blk_op<T, 4>(blocks, op, x, out, odt, rows, n); break;
    default: launch_reduce_blk_op<T, 8>(blocks, op, x, out, odt, rows, n); break;
  }
}
template <typename T>
void launch_reduce_vec(unsigned blocks, int maxv, int op, const T* x, char* out, int odt, int64_t rows, int n) {
  switch (maxv) {
    case 1: launch_reduce_vec_op<T, 1>(blocks, op, x, out, odt, rows, n); break;
    case 2: launch_reduce_vec_op<T, 2>(blocks, op, x, out, odt, rows, n); break;
    case 4: launch_reduce_vec_op<T, 4>(blocks, op, x, out, odt, rows, n); break;
    case 8: launch_reduce_vec_op<T, 8>(blocks, op, x, out, odt, rows, n); break;
    case 12: launch_reduce_vec_op<T, 12>(blocks, op, x, out, odt, rows, n); break;
    case 16: launch_reduce_vec_op<T, 16>(blocks, op, x, out, odt, rows, n); break;
    default: launch_reduce_vec_op<T, 24>(blocks, op, x, out, odt, rows, n); break;
  }
}

#define LC_ROWVEC_DISPATCH6(KERNEL, T, MAXV_RT, BLOCKS, ...)                    \
  switch (MAXV_RT) {                                                           \
    case 1: KERNEL<T, 1><<<BLOCKS, 256, 0, stream()>>>(__VA_ARGS__); break;    \
    case 2: KERNEL<T, 2><<<BLOCKS, 256, 0, stream()>>>(__VA_ARGS__); break;    \
    case 3: KERNEL<T, 3><<<BLOCKS, 256, 0, stream()>>>(__VA_ARGS__); break;    \
    case 4: KERNEL<T, 4><<<BLOCKS, 256, 0, stream()>>>(__VA_ARGS__); break;    \
    case 6: KERNEL<T, 6><<<BLOCKS, 256, 0, stream()>>>(__VA_ARGS__); break;    \
    case 8: KERNEL<T, 8><<<BLOCKS, 256, 0, stream()>>>(__VA_ARGS__); break;    \
    default: KERNEL<T, 12><<<BLOCKS, 256, 0, stream()>>>(__VA_ARGS__); break;  \
  }

#define LC_ROWBLK_DISPATCH(KERNEL, T, MAXV_RT, BLOCKS, ...)                     \
  switch (MAXV_RT) {                                                           \
    case 1: KERNEL<T, 1><<<BLOCKS, 256, 0, stream()>>>(__VA_ARGS__); break;    \
    case 2: KERNEL<T, 2><<<BLOCKS, 256, 0, stream()>>>(__VA_ARGS__); break;    \
    case 4: KERNEL<T, 4><<<BLOCKS, 256, 0, stream()>>>(__VA_ARGS__); break;    \
    default: KERNEL<T, 8><<<BLOCKS, 256, 0, stream()>>>(__VA_ARGS__); break;   \
  }

template <typename CT, typename AT>
void launch_reduce(LcTensor* c, LcTensor* y, int op, Axis3 s) {
  cudaStream_t st = stream();
  if (s.inner == 1) {
    unsigned blocks = blocks_for(s.outer * 32, 256);
    k_reduce_rows<CT, AT><<<blocks, 256, 0, st>>>(c->data(), c->dtype, y->data(), y->dtype, op, s.outer, s.n);
  } else {
    unsigned blocks = blocks_for(s.outer * s.inner, 256);
    k_reduce_cols<CT, AT><<<blocks, 256, 0, st>>>(c->data(), c->dtype, y->data(), y->dtype, op, s.outer, s.n, s.inner);
  }
  LC_LAUNCHED(1);
}

LcTensor* reduce(int op, uint64_t xh, int axis, bool keep, const char* name) {
  LcTensor* x = check(xh, name);
  LC_CHECK(x->ndim >= 1, std::string(name) + ": scalar input");
  int a = norm_axis(axis, x->ndim);
  Axis3 s = split_axis(x, a);
  LC_CHECK(s.n > 0 || op == R_SUM, std::string(name) + ": reduction over an empty axis");
  int odt;
  switch (op) {
    case R_SUM: odt = x->dtype == LC_BOOL ? LC_I32 : x->dtype; break;
    case R_MEAN: odt = x->dtype == LC_F64 ? LC_F64 : LC_F32; break;
    case R_ARGMAX: case R_ARGMIN: odt = LC_I32; break;
    default: odt = x->dtype;
  }
  LcTensor* y = alloc(odt, reduced_shape(x, a, keep));
  if (y->numel() == 0) return y;
  LcTensor* c = contiguous(x);
  int d = x->dtype;
  if (s.inner == 1 && op != R_ARGMAX && op != R_ARGMIN && row_vec_ok(d, s.n, s.outer, 24) && ((uintptr_t)c->data() & 15) == 0) {
    const unsigned blocks = blocks_for(s.outer * 32, 256);
    const int mv = row_vec_maxv(d, s.n);
    const int n = (int)s.n;
    if (d == LC_F16) launch_reduce_vec<__half>(blocks, mv, op, (const __half*)c->data(), y->data(), y->dtype, s.outer, n);
    else if (d == LC_BF16) launch_reduce_vec<__nv_bfloat16>(blocks, mv, op, (const __nv_bfloat16*)c->data(), y->data(), y->dtype, s.outer, n);
    else launch_reduce_vec<float>(blocks, mv, op, (const float*)c->data(), y->data(), y->dtype, s.outer, n);
    LC_LAUNCHED(1);
    if (c != x) release(c);
    return y;
  }
  if (s.inner == 1 && op != R_ARGMAX && op != R_ARGMIN && row_blk_ok(d, s.n, s.outer, c->data())) {
    const unsigned blocks = row_blk_grid(s.outer);
    const int mv = row_blk_maxv(d, s.n);
    const int n = (int)s.n;
    if (d == LC_F16) launch_reduce_blk<__half>(blocks, mv, op, (const __half*)c->data(), y->data(), y->dtype, s.outer, n);
    else if (d == LC_BF16) launch_reduce_blk<__nv_bfloat16>(blocks, mv, op, (const __nv_bfloat16*)c->data(), y->data(), y->dtype, s.outer, n);
    else launch_reduce_blk<float>(blocks, mv, op, (const float*)c->data(), y->data(), y->dtype, s.outer, n);
    LC_LAUNCHED(1);
    if (c != x) release(c);
    return y;
  }
  if (op == R_MEAN) {
    if (d == LC_U64) launch_reduce<uint64_t, double>(c, y, op, s);
    else if (is_float(d)) launch_reduce<double, double>(c, y, op, s);
    else launch_reduce<int64_t, double>(c, y, op, s);
  } else if (d == LC_F64) launch_reduce<double, double>(c, y, op, s);
  else if (is_float(d)) launch_reduce<float, float>(c, y, op, s);
  else if (d == LC_U64) launch_reduce<uint64_t, uint64_t>(c, y, op, s);
  else launch_reduce<int64_t, int64_t>(c, y, op, s);
  if (c != x) release(c);
  return y;
}

}  // namespace

#define RED_ENTRY(fn, op, nm)                                                      \
  int fn(lc_tensor* out, lc_tensor x, int axis, int keep) {                        \
    LC_API_BEGIN *out = handle(reduce(op, x, axis, keep != 0, nm));                \
    LC_API_END                                                                     \
  }

extern "C" {
RED_ENTRY(lc_sum, R_SUM, "sum")
RED_ENTRY(lc_max, R_MAX, "max")
RED_ENTRY(lc_min, R_MIN, "min")
RED_ENTRY(lc_mean, R_MEAN, "mean")
RED_ENTRY(lc_argmax, R_ARGMAX, "argmax")
RED_ENTRY(lc_argmin, R_ARGMIN, "argmin")

int lc_softmax(lc_tensor* out, lc_tensor xh, int axis) {
  LC_API_BEGIN
  LcTensor* x = check(xh, "softmax");
  int a = norm_axis(axis, x->ndim);
  Axis3 s = split_axis(x, a);
  int odt = is_float(x->dtype) ? x->dtype : LC_F32;
  LcTensor* y = alloc(odt, x->dims());
  if (y->numel()) {
    LcTensor* c = contiguous(x);
    cudaStream_t st = stream();
    bool dbl = x->dtype == LC_F64;
    if (s.inner == 1 && odt == x->dtype && row_vec_ok(x->dtype, s.n, s.outer, 12) && (((uintptr_t)c->data() | (uintptr_t)y->data()) & 15) == 0) {
      const unsigned blocks = blocks_for(s.outer * 32, 256);
      // the register tile holds the whole row: sized to it (3 vectors per lane
      // for 768 16-bit values) so short rows keep more warps resident
      const int per = (int)((s.n / (x->dtype == LC_F32 ? 4 : 8) + 31) / 32);
      const int mv = per <= 4 ? per : per <= 6 ? 6 : per <= 8 ? 8 : 12;
      const int n = (int)s.n;
      if (x->dtype == LC_F16) { LC_ROWVEC_DISPATCH6(k_softmax_rows_vec, __half, mv, blocks, (const __half*)c->data(), (__half*)y->data(), s.outer, n) }
      else if (x->dtype == LC_BF16) { LC_ROWVEC_DISPATCH6(k_softmax_rows_vec, __nv_bfloat16, mv, blocks, (const __nv_bfloat16*)c->data(), (__nv_bfloat16*)y->data(), s.outer, n) }
      else { LC_ROWVEC_DISPATCH6(k_softmax_rows_vec, float, mv, blocks, (const float*)c->data(), (float*)y->data(), s.outer, n) }
    } else if (s.inner == 1 && odt == x->dtype && row_blk_ok(x->dtype, s.n, s.outer, c->data()) &&
               ((uintptr_t)y->data() & 15) == 0) {
      const unsigned blocks = row_blk_grid(s.outer);
      const int mv = row_blk_maxv(x->dtype, s.n);
      const int n = (int)s.n;
      if (x->dtype == LC_F16) { LC_ROWBLK_DISPATCH(k_softmax_rows_blk, __half, mv, blocks, (const __half*)c->data(), (__half*)y->data(), s.outer, n) }
      else if (x->dtype == LC_BF16) { LC_ROWBLK_DISPATCH(k_softmax_rows_blk, __nv_bfloat16, mv, blocks, (const __nv_bfloat16*)c->data(), (__nv_bfloat16*)y->data(), s.outer, n) }
      else { LC_ROWBLK_DISPATCH(k_softmax_rows_blk, float, mv, blocks, (const float*)c->data(), (float*)y->data(), s.outer, n) }
    } else if (s.inner == 1) {
      unsigned blocks = blocks_for(s.outer * 32, 256);
      if (dbl) k_softmax_rows<double><<<blocks, 256, 0, st>>>(c->data(), c->dtype, y->data(), odt, s.outer, s.n);
      else k_softmax_rows<float><<<blocks, 256, 0, st>>>(c->data(), c->dtype, y->data(), odt, s.outer, s.n);
    } else {
      unsigned blocks = blocks_for(s.outer * s.inner, 256);
      if (dbl) k_softmax_cols<double><<<blocks, 256, 0, st>>>(c->data(), c->dtype, y->data(), odt, s.outer, s.n, s.inner);
      else k_softmax_cols<float><<<blocks, 256, 0, st>>>(c->data(), c->dtype, y->data(), odt, s.outer, s.n, s.inner);
    }
    LC_LAUNCHED(1);
    if (c != x) release(c);
  }
  *out = handle(y);
  LC_API_END
}

int lc_cumsum(lc_tensor* out, lc_tensor xh, int axis) {
  LC_API_BEGIN
  LcTensor* x = check(xh, "cumsum");
  int a = norm_axis(axis, x->ndim);
  Axis3 s = split_axis(x, a);
  int odt = x->dtype == LC_BOOL ? LC_I32 : x->dtype;
  LcTensor* y = alloc(odt, x->dims());
  if (y->numel()) {
    LcTensor* c = contiguous(x);
    unsigned blocks = blocks_for(s.outer * s.inner, 256);
    cudaStream_t st = stream();
    int d = x->dtype;
    if (d == LC_F64) k_cumsum<double><<<blocks, 256, 0, st>>>(c->data(), d, y->data(), odt, s.outer, s.n, s.inner);
    else if (is_float(d)) k_cumsum<float><<<blocks, 256, 0, st>>>(c->data(), d, y->data(), odt, s.outer, s.n, s.inner);
    else if (d == LC_U64) k_cumsum<uint64_t><<<blocks, 256, 0, st>>>(c->data(), d, y->data(), odt, s.outer, s.n, s.inner);
    else k_cumsum<int64_t><<<blocks, 256, 0, st>>>(c->data(), d, y->data(), odt, s.outer, s.n, s.inner);
    LC_LAUNCHED(1);
    if (c != x) release(c);
  }
  *out = handle(y);
  LC_API_END
}

int lc_sort(lc_tensor* out, lc_tensor xh, int axis) {
  LC_API_BEGIN
  LcTensor* x = check(xh, "sort");
  int r = x->ndim;
  int a = norm_axis(axis, r);
  // move the axis last (a strided view), sort dense rows, then permute back
  std::vector<int64_t> sh, st;
  std::vector<int> perm;
  for (int i = 0; i < r; i++)
    if (i != a) perm.push_back(i);
  perm.push_back(a);
  for (int p : perm) {
    sh.push_back(x->shape[p]);
    st.push_back(x->strides[p]);
  }
  LcTensor* moved = view_of(x, sh, st, x->offset);
  LcTensor* rows = alloc(x->dtype, sh);
  copy_into(moved, rows);
  release(moved);
  int64_t n = x->shape[a], nrows = n ? x->numel() / n : 0;
  if (nrows && n > 1) {
    int P = 1;
    while (P < n) P <<= 1;
    int d = x->dtype;
    size_t esz = (d == LC_F64 || d == LC_U64 || d == LC_I64 || !is_float(d)) ? 8 : 4;
    size_t smem = (size_t)P * esz;
    LC_CHECK(smem <= 96 * 1024, "sort: axis of length " + std::to_string(n) + " is longer than the supported 12288 (8-byte) / 24576 (4-byte) elements");
    cudaStream_t s = stream();
    int threads = P >= 1024 ? 1024 : (P < 32 ? 32 : P);
    if (d == LC_F64) {
      cudaFuncSetAttribute(k_sort_rows<double>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
      k_sort_rows<double><<<(unsigned)nrows, threads, smem, s>>>(rows->data(), d, rows->data(), n, P);
    } else if (is_float(d)) {
      cudaFuncSetAttribute(k_sort_rows<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
      k_sort_rows<float><<<(unsigned)nrows, threads, smem, s>>>(rows->data(), d, rows->data(), n, P);
    } else if (d == LC_U64) {
      cudaFuncSetAttribute(k_sort_rows<uint64_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
      k_sort_rows<uint64_t><<<(unsigned)nrows, threads, smem, s>>>(rows->data(), d, rows->data(), n, P);
    } else {
      cudaFuncSetAttribute(k_sort_rows<int64_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
      k_sort_rows<int64_t><<<(unsigned)nrows, threads, smem, s>>>(rows->data(), d, rows->data(), n, P);
    }
    LC_LAUNCHED(1);
  }
  // inverse permutation back to the input layout
  std::vector<int64_t> bsh(r), bst(r);
  for (int i = 0; i < r; i++) {
    bsh[perm[i]] = rows->shape[i];
    bst[perm[i]] = rows->strides[i];
  }
  LcTensor* back = view_of(rows, bsh, bst, 0);
  LcTensor* y = alloc(x->dtype, x->dims());
  copy_into(back, y);
  release(back);
  release(rows);
  *out = handle(y);
  LC_API_END
}
}  // extern "C"
