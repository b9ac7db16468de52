// Elementwise ops with numpy broadcasting (packages/tensor-backend/src/index.ts:179-198)
// and the optional general numerics (index.ts:265-299).
//
// Two kernel families:
//  * a vectorised fast path (16-byte loads/stores, f32 math) for dense
//    f32/f16/bf16 operands of equal shape, or an [M, N] operand with a
//    row-broadcast [N] operand — the residual adds and the microbench shapes;
//  * a generic strided kernel over broadcast views for everything else
//    (any dtype, rank <= 8), computing in f32 / f64 / int64 / uint64.
#include "lc_api.h"
#include "lc_gelu.cuh"

#include <cmath>
#include <type_traits>

enum EwOp : int {
  OP_ADD, OP_SUB, OP_MUL, OP_DIV, OP_MAX, OP_MIN, OP_POW,
  OP_EQ, OP_NE, OP_LT, OP_LE, OP_GT, OP_GE, OP_AND, OP_OR,
  OP_EXP, OP_LOG, OP_RELU, OP_GELU, OP_SQRT, OP_RSQRT, OP_NEG, OP_ABS, OP_TANH, OP_SIGMOID, OP_ERF, OP_NOT,
  OP_SCALE, OP_COPY
};

// ------------------------------------------------------------- scalar op bodies

__device__ __forceinline__ float gelu_f(float x) { return 0.5f * x * (1.0f + erff(x * 0.7071067811865476f)); }
__device__ __forceinline__ double gelu_d(double x) { return 0.5 * x * (1.0 + erf(x * 0.7071067811865476)); }

template <typename CT>
__device__ __forceinline__ CT bin_op(int op, CT a, CT b) {
  switch (op) {
    case OP_ADD: return a + b;
    case OP_SUB: return a - b;
    case OP_MUL: return a * b;
    case OP_DIV: return a / b;
    case OP_MAX: return a > b ? a : b;
    case OP_MIN: return a < b ? a : b;
    case OP_EQ: return (CT)(a == b);
    case OP_NE: return (CT)(a != b);
    case OP_LT: return (CT)(a < b);
    case OP_LE: return (CT)(a <= b);
    case OP_GT: return (CT)(a > b);
    case OP_GE: return (CT)(a >= b);
    case OP_AND: return (CT)((a != (CT)0) && (b != (CT)0));
    case OP_OR: return (CT)((a != (CT)0) || (b != (CT)0));
  }
  return (CT)0;
}
template <>
__device__ __forceinline__ float bin_op<float>(int op, float a, float b) {
  switch (op) {
    case OP_ADD: return a + b;
    case OP_SUB: return a - b;
    case OP_MUL: return a * b;
    case OP_DIV: return a / b;
    case OP_MAX: return (a > b || isnan(a)) ? a : b;
    case OP_MIN: return (a < b || isnan(a)) ? a : b;
    case OP_POW: return powf(a, b);
    case OP_EQ: return (float)(a == b);
    case OP_NE: return (float)(a != b);
    case OP_LT: return (float)(a < b);
    case OP_LE: return (float)(a <= b);
    case OP_GT: return (float)(a > b);
    case OP_GE: return (float)(a >= b);
    case OP_AND: return (float)((a != 0.f) && (b != 0.f));
    case OP_OR: return (float)((a != 0.f) || (b != 0.f));
  }
  return 0.f;
}
template <>
__device__ __forceinline__ double bin_op<double>(int op, double a, double b) {
  switch (op) {
    case OP_ADD: return a + b;
    case OP_SUB: return a - b;
    case OP_MUL: return a * b;
    case OP_DIV: return a / b;
    case OP_MAX: return (a > b || isnan(a)) ? a : b;
    case OP_MIN: return (a < b || isnan(a)) ? a : b;
    case OP_POW: return pow(a, b);
    case OP_EQ: return (double)(a == b);
    case OP_NE: return (double)(a != b);
    case OP_LT: return (double)(a < b);
    case OP_LE: return (double)(a <= b);
    case OP_GT: return (double)(a > b);
    case OP_GE: return (double)(a >= b);
    case OP_AND: return (double)((a != 0.0) && (b != 0.0));
    case OP_OR: return (double)((a != 0.0) || (b != 0.0));
  }
  return 0.0;
}

template <typename CT>
__device__ __forceinline__ CT un_op(int op, CT x, double s) {
  switch (op) {
    case OP_RELU: return x > (CT)0 ? x : (CT)0;
    case OP_NEG: return (CT)0 - x;
    case OP_ABS: return x < (CT)0 ? (CT)0 - x : x;
    case OP_NOT: return (CT)(x == (CT)0);
    case OP_COPY: return x;
  }
  return x;
}
template <>
__device__ __forceinline__ float un_op<float>(int op, float x, double s) {
  switch (op) {
    case OP_EXP: return expf(x);
    case OP_LOG: return logf(x);
    case OP_RELU: return x > 0.f ? x : (isnan(x) ? x : 0.f);
    case OP_GELU: return gelu_f(x);
    case OP_SQRT: return sqrtf(x);
    case OP_RSQRT: return 1.0f / sqrtf(x);
    case OP_NEG: return -x;
    case OP_ABS: return fabsf(x);
    case OP_TANH: return tanhf(x);
    case OP_SIGMOID: return 1.0f / (1.0f + expf(-x));
    case OP_ERF: return erff(x);
    case OP_NOT: return (float)(x == 0.f);
    case OP_SCALE: return (float)((double)x * s);
    case OP_COPY: return x;
  }
  return x;
}
template <>
__device__ __forceinline__ double un_op<double>(int op, double x, double s) {
  switch (op) {
    case OP_EXP: return exp(x);
    case OP_LOG: return log(x);
    case OP_RELU: return x > 0.0 ? x : (isnan(x) ? x : 0.0);
    case OP_GELU: return gelu_d(x);
    case OP_SQRT: return sqrt(x);
    case OP_RSQRT: return 1.0 / sqrt(x);
    case OP_NEG: return -x;
    case OP_ABS: return fabs(x);
    case OP_TANH: return tanh(x);
    case OP_SIGMOID: return 1.0 / (1.0 + exp(-x));
    case OP_ERF: return erf(x);
    case OP_NOT: return (double)(x == 0.0);
    case OP_SCALE: return x * s;
    case OP_COPY: return x;
  }
  return x;
}

// ------------------------------------------------------------- generic strided kernels

template <typename CT>
__global__ void k_binary(TV a, TV b, char* out, int out_dtype, int op, int64_t n) {
  pdl_trigger();
  pdl_wait();
  LC_GRID_STRIDE(i, n) {
    CT x = ld_as<CT>(a.ptr, a.dtype, tv_offset(a, i));
    CT y = ld_as<CT>(b.ptr, b.dtype, tv_offset(b, i));
    st_as<CT>(out, out_dtype, i, bin_op<CT>(op, x, y));
  }
}

template <typename CT>
__global__ void k_unary(TV a, char* out, int out_dtype, int op, double s, int64_t n) {
  pdl_trigger();
  pdl_wait();
  LC_GRID_STRIDE(i, n) { st_as<CT>(out, out_dtype, i, un_op<CT>(op, ld_as<CT>(a.ptr, a.dtype, tv_offset(a, i)), s)); }
}

template <typename CT>
__global__ void k_where(TV c, TV a, TV b, char* out, int out_dtype, int64_t n) {
  pdl_trigger();
  pdl_wait();
  LC_GRID_STRIDE(i, n) {
    bool cv = ld_as<int64_t>(c.ptr, c.dtype, tv_offset(c, i)) != 0;
    if (c.dtype == LC_F32 || c.dtype == LC_F16 || c.dtype == LC_BF16 || c.dtype == LC_F64)
      cv = ld_as<double>(c.ptr, c.dtype, tv_offset(c, i)) != 0.0;
    CT v = cv ? ld_as<CT>(a.ptr, a.dtype, tv_offset(a, i)) : ld_as<CT>(b.ptr, b.dtype, tv_offset(b, i));
    st_as<CT>(out, out_dtype, i, v);
  }
}

// ------------------------------------------------------------- vectorised fast path

template <typename T> struct Vec;
template <> struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float* v) {
    float4 r = *(const float4*)p;
    v[0] = r.x; v[1] = r.y; v[2] = r.z; v[3] = r.w;
  }
  __device__ static void store(float* p, const float* v) { *(float4*)p = make_float4(v[0], v[1], v[2], v[3]); }
  __device__ static float to_f(float x) { return x; }
  __device__ static float from_f(float x) { return x; }
};
template <> struct Vec<__half> {
  static constexpr int N = 8;
  __device__ static void load(const __half* p, float* v) {
    uint4 r = *(const uint4*)p;
    const __half2* h = (const __half2*)&r;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float2 f = __half22float2(h[i]);
      v[2 * i] = f.x; v[2 * i + 1] = f.y;
    }
  }
  __device__ static void store(__half* p, const float* v) {
    uint4 r;
    __half2* h = (__half2*)&r;
#pragma unroll
    for (int i = 0; i < 4; i++) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    *(uint4*)p = r;
  }
  __device__ static float to_f(__half x) { return __half2float(x); }
  __device__ static __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float* v) {
    uint4 r = *(const uint4*)p;
    const __nv_bfloat162* h = (const __nv_bfloat162*)&r;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x; v[2 * i + 1] = f.y;
    }
  }
  __device__ static void store(__nv_bfloat16* p, const float* v) {
    uint4 r;
    __nv_bfloat162* h = (__nv_bfloat162*)&r;
#pragma unroll
    for (int i = 0; i < 4; i++) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *(uint4*)p = r;
  }
  __device__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

// out[i] = op(a[i], b[i % bn]) over n elements; bn == n for equal shapes,
// bn == N (row length) for a row-broadcast operand. n and bn are multiples of V::N.
template <typename T, int OP>
__global__ void __launch_bounds__(256) k_vec_binary(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ out, int64_t n, int64_t bn) {
  pdl_trigger();
  pdl_wait();
  using V = Vec<T>;
  const int64_t nv = n / V::N;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += (int64_t)gridDim.x * blockDim.x) {
    int64_t i = v * V::N;
    float x[V::N], y[V::N];
    V::load(a + i, x);
    V::load(b + (bn == n ? i : i % bn), y);
#pragma unroll
    for (int j = 0; j < V::N; j++) x[j] = bin_op<float>(OP, x[j], y[j]);
    V::store(out + i, x);
  }
}

template <typename T, int OP>
__global__ void __launch_bounds__(256) k_vec_unary(const T* __restrict__ a, T* __restrict__ out, int64_t n, float s) {
  pdl_trigger();
  pdl_wait();
  using V = Vec<T>;
  const int64_t nv = n / V::N;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += (int64_t)gridDim.x * blockDim.x) {
    int64_t i = v * V::N;
    float x[V::N];
    V::load(a + i, x);
    if constexpr (OP == OP_GELU && sizeof(T) == 2) {
      // stored in 16 bits: erf by Abramowitz & Stegun 7.1.26 (|error| <= 1.5e-7), packed pairs
#pragma unroll
      for (int j = 0; j < V::N; j += 2) {
        const float2 g = gelu_as2(make_float2(x[j], x[j + 1]));
        x[j] = g.x;
        x[j + 1] = g.y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < V::N; j++) x[j] = (OP == OP_SCALE) ? x[j] * s : un_op<float>(OP, x[j], 0.0);
    }
    V::store(out + i, x);
  }
}

using namespace lc;

namespace {

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

template <typename T>
bool try_vec_binary(int op, LcTensor* a, LcTensor* b, LcTensor* y) {
  using V = Vec<T>;
  int64_t n = y->numel();
  if (!a->contiguous() || !b->contiguous() || n % V::N) return false;
  if (!aligned16(a->data()) || !aligned16(b->data()) || !aligned16(y->data())) return false;
  int64_t bn;
  if (b->numel() == n && a->numel() == n) bn = n;
  else if (a->numel() == n && y->ndim >= 1 && b->numel() == y->shape[y->ndim - 1] &&
           (b->ndim == 1 || (b->ndim >= 1 && b->shape[b->ndim - 1] == b->numel()))) bn = b->numel();
  else return false;
  if (bn % V::N) return false;
  unsigned blocks = blocks_for(n / V::N, 256);
  const T* pa = (const T*)a->data();
  const T* pb = (const T*)b->data();
  T* po = (T*)y->data();
  cudaStream_t st = stream();
  switch (op) {
    case OP_ADD: lc::launch_chain(k_vec_binary<T, OP_ADD>, dim3(blocks), dim3(256), 0, st, pa, pb, po, n, bn); break;
    case OP_SUB: lc::launch_chain(k_vec_binary<T, OP_SUB>, dim3(blocks), dim3(256), 0, st, pa, pb, po, n, bn); break;
    case OP_MUL: lc::launch_chain(k_vec_binary<T, OP_MUL>, dim3(blocks), dim3(256), 0, st, pa, pb, po, n, bn); break;
    case OP_DIV: lc::launch_chain(k_vec_binary<T, OP_DIV>, dim3(blocks), dim3(256), 0, st, pa, pb, po, n, bn); break;
    case OP_MAX: lc::launch_chain(k_vec_binary<T, OP_MAX>, dim3(blocks), dim3(256), 0, st, pa, pb, po, n, bn); break;
    default: return false;
  }
  LC_LAUNCHED(1);
  return true;
}

template <typename T>
bool try_vec_unary(int op, LcTensor* a, LcTensor* y, double s) {
  using V = Vec<T>;
  int64_t n = y->numel();
  if (!a->contiguous() || n % V::N || !aligned16(a->data()) || !aligned16(y->data())) return false;
  unsigned blocks = blocks_for(n / V::N, 256);
  const T* pa = (const T*)a->data();
  T* po = (T*)y->data();
  cudaStream_t st = stream();
  switch (op) {
    case OP_EXP: lc::launch_chain(k_vec_unary<T, OP_EXP>, dim3(blocks), dim3(256), 0, st, pa, po, n, 0.f); break;
    case OP_RELU: lc::launch_chain(k_vec_unary<T, OP_RELU>, dim3(blocks), dim3(256), 0, st, pa, po, n, 0.f); break;
    case OP_GELU: lc::launch_chain(k_vec_unary<T, OP_GELU>, dim3(blocks), dim3(256), 0, st, pa, po, n, 0.f); break;
    case OP_SCALE:
      if (std::is_same<T, float>::value) return false;  // f32 scale keeps double math in the generic path
      lc::launch_chain(k_vec_unary<T, OP_SCALE>, dim3(blocks), dim3(256), 0, st, pa, po, n, (float)s); break;
    default: return false;
  }
  LC_LAUNCHED(1);
  return true;
}

// Compute type: 0 float, 1 int64, 2 double, 3 uint64
int ctype_of(int d1, int d2) {
  if (d1 == LC_F64 || d2 == LC_F64) return 2;
  bool f1 = is_float(d1), f2 = is_float(d2);
  if (f1 && f2) return 0;
  if (f1 || f2) return 2;  // float with integer: compare/compute exactly in double
  if (d1 == LC_U64 || d2 == LC_U64) return 3;
  return 1;
}

bool is_cmp(int op) { return op >= OP_EQ && op <= OP_OR; }

LcTensor* binary(int op, uint64_t ah, uint64_t bh, const char* name) {
  LcTensor* a = check(ah, name);
  LcTensor* b = check(bh, name);
  std::vector<int64_t> sh = broadcast_shapes({a->dims(), b->dims()});
  int odt;
  if (is_cmp(op)) odt = LC_BOOL;
  else if (op == OP_DIV || op == OP_POW) {
    odt = promote(a->dtype, b->dtype);
    if (!is_float(odt)) odt = LC_F32;
  } else {
    odt = promote(a->dtype, b->dtype);
  }
  if (op == OP_DIV) LC_CHECK(a->dtype != LC_U64 && a->dtype != LC_I64 && b->dtype != LC_U64 && b->dtype != LC_I64,
                            "div: u64/i64 are not accepted (cast to a float dtype first)");
  LcTensor* y = alloc(odt, sh);
  int64_t n = y->numel();
  if (n == 0) return y;
  if (a->dtype == b->dtype && a->dtype == odt) {
    bool done = false;
    if (odt == LC_F32) done = try_vec_binary<float>(op, a, b, y);
    else if (odt == LC_F16) done = try_vec_binary<__half>(op, a, b, y);
    else if (odt == LC_BF16) done = try_vec_binary<__nv_bfloat16>(op, a, b, y);
    if (done) return y;
  }
  TV va = tv_broadcast(a, sh), vb = tv_broadcast(b, sh);
  int ct = ctype_of(a->dtype, b->dtype);
  if (op == OP_DIV || op == OP_POW) ct = (ct == 2 || odt == LC_F64) ? 2 : (ct == 0 ? 0 : 2);
  unsigned blocks = blocks_for(n, 256);
  cudaStream_t st = stream();
  switch (ct) {
    case 0: lc::launch_chain(k_binary<float>, dim3(blocks), dim3(256), 0, st, va, vb, y->data(), odt, op, n); break;
    case 1: lc::launch_chain(k_binary<int64_t>, dim3(blocks), dim3(256), 0, st, va, vb, y->data(), odt, op, n); break;
    case 2: lc::launch_chain(k_binary<double>, dim3(blocks), dim3(256), 0, st, va, vb, y->data(), odt, op, n); break;
    default: lc::launch_chain(k_binary<uint64_t>, dim3(blocks), dim3(256), 0, st, va, vb, y->data(), odt, op, n); break;
  }
  LC_LAUNCHED(1);
  return y;
}

// float-valued unary ops keep float dtypes and map integers to f32
bool float_valued(int op) {
  return op == OP_EXP || op == OP_LOG || op == OP_GELU || op == OP_SQRT || op == OP_RSQRT || op == OP_TANH ||
         op == OP_SIGMOID || op == OP_ERF || op == OP_SCALE;
}

LcTensor* unary(int op, uint64_t xh, const char* name, double s = 0.0) {
  LcTensor* x = check(xh, name);
  int odt;
  if (op == OP_NOT) odt = LC_BOOL;
  else if (float_valued(op)) odt = is_float(x->dtype) ? x->dtype : LC_F32;
  else if ((op == OP_NEG || op == OP_ABS) && x->dtype == LC_BOOL) odt = LC_I32;
  else odt = x->dtype;
  LcTensor* y = alloc(odt, x->dims());
  int64_t n = y->numel();
  if (n == 0) return y;
  if (x->dtype == odt) {
    bool done = false;
    if (odt == LC_F32) done = try_vec_unary<float>(op, x, y, s);
    else if (odt == LC_F16) done = try_vec_unary<__half>(op, x, y, s);
    else if (odt == LC_BF16) done = try_vec_unary<__nv_bfloat16>(op, x, y, s);
    if (done) return y;
  }
  TV vx = tv(x);
  int ct;
  if (x->dtype == LC_F64) ct = 2;
  else if (is_float(x->dtype)) ct = (op == OP_SCALE) ? 2 : 0;
  else if (float_valued(op)) ct = 2;
  else if (x->dtype == LC_U64) ct = 3;
  else ct = 1;
  unsigned blocks = blocks_for(n, 256);
  cudaStream_t st = stream();
  switch (ct) {
    case 0: lc::launch_chain(k_unary<float>, dim3(blocks), dim3(256), 0, st, vx, y->data(), odt, op, s, n); break;
    case 1: lc::launch_chain(k_unary<int64_t>, dim3(blocks), dim3(256), 0, st, vx, y->data(), odt, op, s, n); break;
    case 2: lc::launch_chain(k_unary<double>, dim3(blocks), dim3(256), 0, st, vx, y->data(), odt, op, s, n); break;
    default: lc::launch_chain(k_unary<uint64_t>, dim3(blocks), dim3(256), 0, st, vx, y->data(), odt, op, s, n); break;
  }
  LC_LAUNCHED(1);
  return y;
}

}  // namespace

// Converting copy into a strided destination (used by concat).
template <typename CT>
__global__ void k_copy_to_strided(TV src, TV dst, int64_t n) {
  pdl_trigger();
  pdl_wait();
  LC_GRID_STRIDE(i, n) { st_as<CT>(dst.ptr, dst.dtype, tv_offset(dst, i), ld_as<CT>(src.ptr, src.dtype, tv_offset(src, i))); }
}

void lc_internal_copy_strided(const LcTensor* src, LcTensor* dst) {
  int64_t n = src->numel();
  if (!n) return;
  TV s = tv(src), d = tv(dst);
  unsigned blocks = blocks_for(n, 256);
  int ct = ctype_of(src->dtype, dst->dtype);
  if (src->dtype == LC_U64 || dst->dtype == LC_U64) ct = 3;
  if (is_float(src->dtype) && !is_float(dst->dtype)) ct = 2;
  switch (ct) {
    case 0: lc::launch_chain(k_copy_to_strided<float>, dim3(blocks), dim3(256), 0, stream(), s, d, n); break;
    case 1: lc::launch_chain(k_copy_to_strided<int64_t>, dim3(blocks), dim3(256), 0, stream(), s, d, n); break;
    case 2: lc::launch_chain(k_copy_to_strided<double>, dim3(blocks), dim3(256), 0, stream(), s, d, n); break;
    default: lc::launch_chain(k_copy_to_strided<uint64_t>, dim3(blocks), dim3(256), 0, stream(), s, d, n); break;
  }
  LC_LAUNCHED(1);
}

#define BIN_ENTRY(fn, op, nm)                                    \
  int fn(lc_tensor* out, lc_tensor a, lc_tensor b) {             \
    LC_API_BEGIN *out = handle(binary(op, a, b, nm));            \
    LC_API_END                                                   \
  }
#define UN_ENTRY(fn, op, nm)                                     \
  int fn(lc_tensor* out, lc_tensor x) {                          \
    LC_API_BEGIN *out = handle(unary(op, x, nm));                \
    LC_API_END                                                   \
  }

extern "C" {
BIN_ENTRY(lc_add, OP_ADD, "add")
BIN_ENTRY(lc_sub, OP_SUB, "sub")
BIN_ENTRY(lc_mul, OP_MUL, "mul")
BIN_ENTRY(lc_div, OP_DIV, "div")
BIN_ENTRY(lc_maximum, OP_MAX, "maximum")
BIN_ENTRY(lc_pow, OP_POW, "pow")
BIN_ENTRY(lc_equal, OP_EQ, "equal")
BIN_ENTRY(lc_not_equal, OP_NE, "notEqual")
BIN_ENTRY(lc_less, OP_LT, "less")
BIN_ENTRY(lc_less_equal, OP_LE, "lessEqual")
BIN_ENTRY(lc_greater, OP_GT, "greater")
BIN_ENTRY(lc_greater_equal, OP_GE, "greaterEqual")
BIN_ENTRY(lc_logical_and, OP_AND, "logicalAnd")
BIN_ENTRY(lc_logical_or, OP_OR, "logicalOr")
UN_ENTRY(lc_exp, OP_EXP, "exp")
UN_ENTRY(lc_log, OP_LOG, "log")
UN_ENTRY(lc_relu, OP_RELU, "relu")
UN_ENTRY(lc_gelu, OP_GELU, "gelu")
UN_ENTRY(lc_sqrt, OP_SQRT, "sqrt")
UN_ENTRY(lc_rsqrt, OP_RSQRT, "rsqrt")
UN_ENTRY(lc_neg, OP_NEG, "neg")
UN_ENTRY(lc_abs, OP_ABS, "abs")
UN_ENTRY(lc_tanh, OP_TANH, "tanh")
UN_ENTRY(lc_sigmoid, OP_SIGMOID, "sigmoid")
UN_ENTRY(lc_erf, OP_ERF, "erf")
UN_ENTRY(lc_logical_not, OP_NOT, "logicalNot")

int lc_scale(lc_tensor* out, lc_tensor x, double s) {
  LC_API_BEGIN *out = handle(unary(OP_SCALE, x, "scale", s));
  LC_API_END
}

int lc_where(lc_tensor* out, lc_tensor ch, lc_tensor ah, lc_tensor bh) {
  LC_API_BEGIN
  LcTensor* c = check(ch, "where");
  LcTensor* a = check(ah, "where");
  LcTensor* b = check(bh, "where");
  std::vector<int64_t> sh = broadcast_shapes({c->dims(), a->dims(), b->dims()});
  int odt = promote(a->dtype, b->dtype);
  LcTensor* y = alloc(odt, sh);
  int64_t n = y->numel();
  if (n) {
    TV vc = tv_broadcast(c, sh), va = tv_broadcast(a, sh), vb = tv_broadcast(b, sh);
    unsigned blocks = blocks_for(n, 256);
    int ct = ctype_of(a->dtype, b->dtype);
    if (odt == LC_U64) ct = 3;
    switch (ct) {
      case 0: lc::launch_chain(k_where<float>, dim3(blocks), dim3(256), 0, stream(), vc, va, vb, y->data(), odt, n); break;
      case 1: lc::launch_chain(k_where<int64_t>, dim3(blocks), dim3(256), 0, stream(), vc, va, vb, y->data(), odt, n); break;
      case 2: lc::launch_chain(k_where<double>, dim3(blocks), dim3(256), 0, stream(), vc, va, vb, y->data(), odt, n); break;
      default: lc::launch_chain(k_where<uint64_t>, dim3(blocks), dim3(256), 0, stream(), vc, va, vb, y->data(), odt, n); break;
    }
    LC_LAUNCHED(1);
  }
  *out = handle(y);
  LC_API_END
}
}  // extern "C"
