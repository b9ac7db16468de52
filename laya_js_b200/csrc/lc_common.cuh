// Shared definitions of liblaya_cuda: dtypes, the tensor handle, error slot,
// device-side typed loads/stores.
//
// A tensor handle is a pointer to an LcTensor: a strided view (shape,
// element strides, element offset) over a reference-counted device Storage.
// reshape/transpose/slice/split only make new views; kernels that need dense
// input call lc::contiguous() first. This mirrors what the reference
// contract requires (packages/tensor-backend/src/index.ts:168-177: numpy
// view/copy semantics) without materialising permutes on the hot path.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdexcept>
#include <string>
#include <vector>

#define LC_MAX_DIMS 8

enum LcDType : int {
  LC_F32 = 0, LC_F16 = 1, LC_BF16 = 2, LC_I32 = 3, LC_BOOL = 4, LC_U8 = 5, LC_I8 = 6,
  LC_U16 = 7, LC_I16 = 8, LC_U32 = 9, LC_U64 = 10, LC_I64 = 11, LC_F64 = 12, LC_NUM_DTYPES = 13
};

inline int dtype_size(int d) {
  switch (d) {
    case LC_F32: case LC_I32: case LC_U32: return 4;
    case LC_F16: case LC_BF16: case LC_U16: case LC_I16: return 2;
    case LC_BOOL: case LC_U8: case LC_I8: return 1;
    case LC_U64: case LC_I64: case LC_F64: return 8;
  }
  throw std::runtime_error("unknown dtype " + std::to_string(d));
}
inline bool is_float(int d) { return d == LC_F32 || d == LC_F16 || d == LC_BF16 || d == LC_F64; }
inline bool is_half(int d) { return d == LC_F16 || d == LC_BF16; }
inline bool is_signed_int(int d) { return d == LC_I32 || d == LC_I8 || d == LC_I16 || d == LC_I64; }
const char* dtype_name(int d);

struct LcStorage {
  void* ptr = nullptr;
  size_t bytes = 0;
  int refs = 1;
  bool external = false;  // not owned (never freed by the library)
  // The launch count when lc_from_host filled it, -1 once lc_copy_into has
  // written it (or for memory it did not upload): a weight no kernel writes.
  int64_t upload_mark = -1;
  uint64_t id = 0;       // unique per storage for the process's lifetime
  uint32_t version = 0;  // bumped whenever lc_copy_into writes it
};

struct LcTensor {
  uint64_t magic;
  LcStorage* st;
  int dtype;
  int ndim;
  int64_t shape[LC_MAX_DIMS];
  int64_t strides[LC_MAX_DIMS];
  int64_t offset;  // elements

  int64_t numel() const {
    int64_t n = 1;
    for (int i = 0; i < ndim; i++) n *= shape[i];
    return n;
  }
  bool contiguous() const {
    int64_t s = 1;
    for (int i = ndim - 1; i >= 0; i--) {
      if (shape[i] != 1 && strides[i] != s) return false;
      s *= shape[i];
    }
    return true;
  }
  char* data() const { return (char*)st->ptr + offset * dtype_size(dtype); }
  std::vector<int64_t> dims() const { return std::vector<int64_t>(shape, shape + ndim); }
};

// Strided view passed by value to kernels.
struct TV {
  char* ptr;
  int dtype;
  int ndim;
  int64_t shape[LC_MAX_DIMS];
  int64_t strides[LC_MAX_DIMS];
};

namespace lc {

struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};
[[noreturn]] inline void fail(const std::string& m) { throw Error(m); }
#define LC_CHECK(cond, msg)                          \
  do {                                               \
    if (!(cond)) ::lc::fail(std::string(msg));       \
  } while (0)
void cuda_check(cudaError_t e, const char* what);
#define CUDA_OK(x) ::lc::cuda_check((x), #x)

cudaStream_t stream();
int device();
int num_sms();
void* dmalloc(size_t bytes);
void dfree(void* p);

// Tensor construction / lookup (all handles are validated against the live set).
LcTensor* check(uint64_t h, const char* what = "tensor");
LcTensor* alloc(int dtype, const std::vector<int64_t>& shape);
LcTensor* view_of(const LcTensor* x, const std::vector<int64_t>& shape, const std::vector<int64_t>& strides, int64_t offset);
LcTensor* contiguous(LcTensor* x);  // returns x itself (refcount unchanged) when already dense; else a new dense copy
void release(LcTensor* t);           // frees a temporary made inside an op
uint64_t handle(LcTensor* t);
TV tv(const LcTensor* t);
TV tv_broadcast(const LcTensor* t, const std::vector<int64_t>& out_shape);  // numpy-broadcast strides
std::vector<int64_t> broadcast_shapes(const std::vector<std::vector<int64_t>>& shapes);
int promote(int a, int b);
int norm_axis(int axis, int ndim);
std::string shape_str(const std::vector<int64_t>& s);
void copy_into(const LcTensor* src, LcTensor* dst_dense);  // strided copy + dtype conversion into a dense tensor
inline unsigned blocks_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  int64_t cap = (int64_t)num_sms() * 32;
  return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

// Programmatic dependent launch for a chain of kernels on one stream (the
// fused encoder's forward): while a PdlScope lives on the calling thread,
// launch_chain() lets each kernel launch before its predecessor has finished.
// Only kernels that call pdl_wait() in every CTA before touching memory an
// earlier kernel wrote (and before exiting) may be launched this way.
bool& pdl_flag();
// The storage was filled by a host upload, no kernel has written it since,
// and a kernel has been launched after the upload (so the copy has landed
// before any later kernel starts): a GEMM may read it before pdl_wait().
bool upload_settled(const LcStorage* st);
// Called once a storage's memory is released: drops derived data cached for
// it (the packed attention masks).
void storage_released(uint64_t id);
// Called while a capture ends (aborted: after the capture, whose allocations
// no longer exist): releases data cached during the capture.
void capture_ending(bool aborted);
// A CUDA graph capture (lc_graph_capture_begin) is in progress.
bool capturing();
struct PdlScope {
  bool prev;
  PdlScope() : prev(pdl_flag()) { pdl_flag() = true; }
  ~PdlScope() { pdl_flag() = prev; }
  PdlScope(const PdlScope&) = delete;
  PdlScope& operator=(const PdlScope&) = delete;
};
// Launch attributes for a kernel of the chain: the caller's (e.g. a cluster
// size) plus programmatic stream serialisation when a PdlScope is active.
inline void chain_attrs(cudaLaunchConfig_t& cfg, cudaLaunchAttribute* at, int n_given) {
  int n = n_given;
  if (pdl_flag()) {
    at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[n].val.programmaticStreamSerializationAllowed = 1;
    n++;
  }
  cfg.attrs = n ? at : nullptr;
  cfg.numAttrs = (unsigned)n;
}
template <typename... KArgs, typename... Args>
void launch_chain(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  chain_attrs(cfg, at, 0);
  CUDA_OK(cudaLaunchKernelEx(&cfg, kernel, args...));
}

}  // namespace lc

// The device side of programmatic dependent launch. pdl_trigger(): this CTA
// no longer holds back the launch of the next kernel of the chain.
// pdl_wait(): returns once the kernels this one depends on have completed
// and their memory is visible (at once when launched without the attribute).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------- device helpers

// f32 <-> f32 / f16 / bf16 element (round to nearest even into 16 bits)
template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename CT>
__device__ __forceinline__ CT ld_as(const char* p, int dtype, int64_t i) {
  switch (dtype) {
    case LC_F32: return (CT)((const float*)p)[i];
    case LC_F16: return (CT)__half2float(((const __half*)p)[i]);
    case LC_BF16: return (CT)__bfloat162float(((const __nv_bfloat16*)p)[i]);
    case LC_I32: return (CT)((const int32_t*)p)[i];
    case LC_BOOL: return (CT)(((const uint8_t*)p)[i] != 0);
    case LC_U8: return (CT)((const uint8_t*)p)[i];
    case LC_I8: return (CT)((const int8_t*)p)[i];
    case LC_U16: return (CT)((const uint16_t*)p)[i];
    case LC_I16: return (CT)((const int16_t*)p)[i];
    case LC_U32: return (CT)((const uint32_t*)p)[i];
    case LC_U64: return (CT)((const uint64_t*)p)[i];
    case LC_I64: return (CT)((const int64_t*)p)[i];
    case LC_F64: return (CT)((const double*)p)[i];
  }
  return (CT)0;
}

// Float -> integer conversion truncates toward zero (C semantics), saturating
// nothing: out-of-range values are undefined in the contract, so we clamp to
// keep the conversion well defined on the device.
template <typename IT, typename CT>
__device__ __forceinline__ IT to_int(CT v) {
  return (IT)v;
}

template <typename CT>
__device__ __forceinline__ void st_as(char* p, int dtype, int64_t i, CT v) {
  switch (dtype) {
    case LC_F32: ((float*)p)[i] = (float)v; break;
    case LC_F16: ((__half*)p)[i] = __float2half_rn((float)v); break;
    case LC_BF16: ((__nv_bfloat16*)p)[i] = __float2bfloat16_rn((float)v); break;
    case LC_I32: ((int32_t*)p)[i] = (int32_t)(int64_t)v; break;
    case LC_BOOL: ((uint8_t*)p)[i] = (v != (CT)0) ? 1 : 0; break;
    case LC_U8: ((uint8_t*)p)[i] = (uint8_t)(int64_t)v; break;
    case LC_I8: ((int8_t*)p)[i] = (int8_t)(int64_t)v; break;
    case LC_U16: ((uint16_t*)p)[i] = (uint16_t)(int64_t)v; break;
    case LC_I16: ((int16_t*)p)[i] = (int16_t)(int64_t)v; break;
    case LC_U32: ((uint32_t*)p)[i] = (uint32_t)(int64_t)v; break;
    case LC_U64: ((uint64_t*)p)[i] = (uint64_t)v; break;
    case LC_I64: ((int64_t*)p)[i] = (int64_t)v; break;
    case LC_F64: ((double*)p)[i] = (double)v; break;
  }
}

// Offset (elements) of the element with linear index `li` of a broadcast view.
__device__ __forceinline__ int64_t tv_offset(const TV& t, int64_t li) {
  int64_t off = 0;
  for (int d = t.ndim - 1; d >= 0; d--) {
    int64_t s = t.shape[d];
    int64_t c = li % s;
    li /= s;
    off += c * t.strides[d];
  }
  return off;
}

#define LC_GRID_STRIDE(i, n) \
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (n); i += (int64_t)gridDim.x * blockDim.x)
