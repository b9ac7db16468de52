// liblaya_cuda core: library state, stream-ordered allocation, the live
// handle registry, transfers, views and dtype-converting copies.
//
// Replaces the lifetime half of the reference contract
// (packages/tensor-backend/src/index.ts:145-177): fromHost/read/dispose/
// flush/destroy and reshape/transpose/slice/split/concat/cast.
#include "lc_common.cuh"
#include "lc_api.h"
#include "lc_gemm.h"

#include <algorithm>
#include <cstring>
#include <memory>
#include <mutex>
#include <unordered_map>
#include <unordered_set>
#include <thread>
#include <vector>

static const uint64_t kMagic = 0x4c41594143554441ull;  // "LAYACUDA"

namespace {
struct State {
  bool inited = false;
  int device = 0;
  int sms = 148;
  cudaStream_t own = nullptr;
  cudaStream_t cur = nullptr;
  std::unordered_set<LcTensor*> live;
  int64_t live_bytes = 0;
  int64_t launches = 0;
  // stream capture (lc_graph_capture_*): allocations made while capturing
  // become the graph's own (alloc nodes, freed by free nodes inside it);
  // memory that existed before the capture and is released during it stays
  // allocated until the graph is destroyed, since its kernels may read it.
  int64_t alloc_cap = 0;  // lc_debug_set_alloc_cap: tensor bytes allowed at once (0 = no cap)
  bool capturing = false;
  std::unordered_set<void*> cap_allocs;
  std::vector<void*> cap_deferred;
  uint64_t next_storage_id = 0;
};
State& S() {
  static State s;
  return s;
}
thread_local std::string g_err;
}  // namespace

const char* dtype_name(int d) {
  static const char* n[] = {"f32", "f16", "bf16", "i32", "bool", "u8", "i8", "u16", "i16", "u32", "u64", "i64", "f64"};
  return (d >= 0 && d < LC_NUM_DTYPES) ? n[d] : "?";
}

namespace lc {

void set_error(const std::string& m) { g_err = m; }

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    fail(std::string("CUDA error ") + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ") in " + what);
  }
}

static void ensure_init() {
  if (!S().inited) fail("liblaya_cuda: lc_init(device) was not called");
}

cudaStream_t stream() { return S().cur; }
int device() { return S().device; }
int num_sms() { return S().sms; }
void count_launch(int n) { S().launches += n; }
bool capturing() { return S().capturing; }
bool upload_settled(const LcStorage* st) { return st->upload_mark >= 0 && S().launches > st->upload_mark; }
// The fused encoder chains its kernels with programmatic dependent launch
// (a PdlScope). The contract's ops are launched serialised unless
// LAYA_CUDA_PDL=1: every kernel launched through launch_chain waits for its
// predecessor before touching memory, but with chaining on, a padded 4-bit
// contract forward gave a 1024-token prompt's hidden rows that differed from
// one process to the next (up to 5.4e-2 from the CPU reference, against
// 1.1e-2 serialised, which is the same in every run; the ordering is not yet
// found), and chaining made the padded 256-prompt forward slower, not faster
// (71-72 ms against 65-68 ms).
bool& pdl_flag() {
  static const bool dflt = [] {
    const char* v = getenv("LAYA_CUDA_PDL");
    return v && v[0] == '1';
  }();
  static thread_local bool on = dflt;
  return on;
}

void* dmalloc(size_t bytes) {
  ensure_init();
  void* p = nullptr;
  if (bytes == 0) bytes = 16;
  bytes = (bytes + 255) & ~(size_t)255;
  cudaError_t e = cudaMallocAsync(&p, bytes, S().cur);
  if (e != cudaSuccess) {
    cudaGetLastError();
    fail("out of device memory allocating " + std::to_string(bytes) + " bytes (" + cudaGetErrorString(e) + ")");
  }
  if (S().capturing) S().cap_allocs.insert(p);
  return p;
}
void dfree(void* p) {
  if (!p) return;
  State& s = S();
  if (s.capturing) {
    if (!s.cap_allocs.erase(p)) {
      s.cap_deferred.push_back(p);
      return;
    }
  }
  cudaFreeAsync(p, s.cur);
}

LcTensor* check(uint64_t h, const char* what) {
  ensure_init();
  LcTensor* t = reinterpret_cast<LcTensor*>(h);
  if (!h) fail(std::string(what) + ": null tensor handle");
  if (!S().live.count(t) || t->magic != kMagic) fail(std::string(what) + ": tensor used after dispose (or not a tensor handle)");
  return t;
}

static LcTensor* new_tensor(LcStorage* st, int dtype, const std::vector<int64_t>& shape) {
  LC_CHECK(shape.size() <= LC_MAX_DIMS, "rank above 8 is not supported");
  LcTensor* t = new LcTensor();
  t->magic = kMagic;
  t->st = st;
  t->dtype = dtype;
  t->ndim = (int)shape.size();
  int64_t s = 1;
  for (int i = t->ndim - 1; i >= 0; i--) {
    LC_CHECK(shape[i] >= 0, "negative dimension");
    t->shape[i] = shape[i];
    t->strides[i] = s;
    s *= shape[i];
  }
  t->offset = 0;
  S().live.insert(t);
  return t;
}

LcTensor* alloc(int dtype, const std::vector<int64_t>& shape) {
  int64_t n = 1;
  for (auto d : shape) n *= d;
  const size_t bytes = (size_t)n * dtype_size(dtype);
  if (S().alloc_cap && S().live_bytes + (int64_t)bytes > S().alloc_cap)
    fail("out of device memory allocating " + std::to_string(bytes) + " bytes (the allocation cap of " +
         std::to_string(S().alloc_cap) + " bytes would be exceeded)");
  LcStorage* st = new LcStorage();
  st->id = ++S().next_storage_id;
  st->bytes = bytes;
  st->ptr = dmalloc(st->bytes);
  S().live_bytes += (int64_t)st->bytes;
  return new_tensor(st, dtype, shape);
}

LcTensor* view_of(const LcTensor* x, const std::vector<int64_t>& shape, const std::vector<int64_t>& strides, int64_t offset) {
  LcTensor* t = new_tensor(x->st, x->dtype, shape);
  x->st->refs++;
  for (int i = 0; i < t->ndim; i++) t->strides[i] = strides[i];
  t->offset = offset;
  return t;
}

void release(LcTensor* t) {
  if (!t || !S().live.count(t)) return;
  S().live.erase(t);
  t->magic = 0;
  if (--t->st->refs == 0) {
    storage_released(t->st->id);
    if (!t->st->external) {
      dfree(t->st->ptr);
      S().live_bytes -= (int64_t)t->st->bytes;
    }
    delete t->st;
  }
  delete t;
}

uint64_t handle(LcTensor* t) { return reinterpret_cast<uint64_t>(t); }

TV tv(const LcTensor* t) {
  TV v;
  v.ptr = (char*)t->st->ptr + t->offset * dtype_size(t->dtype);
  v.dtype = t->dtype;
  v.ndim = t->ndim;
  for (int i = 0; i < t->ndim; i++) {
    v.shape[i] = t->shape[i];
    v.strides[i] = t->strides[i];
  }
  return v;
}

TV tv_broadcast(const LcTensor* t, const std::vector<int64_t>& out) {
  TV v;
  v.ptr = (char*)t->st->ptr + t->offset * dtype_size(t->dtype);
  v.dtype = t->dtype;
  v.ndim = (int)out.size();
  int lead = v.ndim - t->ndim;
  LC_CHECK(lead >= 0, "broadcast: input rank above output rank");
  for (int i = 0; i < v.ndim; i++) {
    v.shape[i] = out[i];
    if (i < lead) {
      v.strides[i] = 0;
    } else {
      int64_t d = t->shape[i - lead];
      LC_CHECK(d == out[i] || d == 1, "broadcast: incompatible shapes");
      v.strides[i] = (d == 1 && out[i] != 1) ? 0 : t->strides[i - lead];
    }
  }
  return v;
}

std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); i++) r += (i ? "," : "") + std::to_string(s[i]);
  return r + "]";
}

std::vector<int64_t> broadcast_shapes(const std::vector<std::vector<int64_t>>& shapes) {
  size_t r = 0;
  for (auto& s : shapes) r = std::max(r, s.size());
  std::vector<int64_t> out(r, 1);
  for (auto& s : shapes) {
    size_t lead = r - s.size();
    for (size_t i = 0; i < s.size(); i++) {
      int64_t d = s[i];
      int64_t& o = out[lead + i];
      if (o == 1) o = d;
      else if (d != 1 && d != o) {
        std::string m = "shapes do not broadcast:";
        for (auto& x : shapes) m += " " + shape_str(x);
        fail(m);
      }
    }
  }
  return out;
}

int promote(int a, int b) {
  if (a == b) return a;
  bool fa = is_float(a), fb = is_float(b);
  if (fa || fb) {
    if (a == LC_F64 || b == LC_F64) return LC_F64;
    if (fa && fb) return LC_F32;  // f16+bf16, f16+f32, bf16+f32
    return fa ? a : b;            // float with an integer keeps the float dtype
  }
  if (a == LC_BOOL) return b;
  if (b == LC_BOOL) return a;
  int sa = dtype_size(a), sb = dtype_size(b);
  bool ua = !is_signed_int(a), ub = !is_signed_int(b);
  if (ua == ub) return sa >= sb ? a : b;
  // mixed signedness: the signed type if it is wider, else the next wider signed type
  int s = ua ? b : a, u = ua ? a : b;
  if (dtype_size(s) > dtype_size(u)) return s;
  switch (dtype_size(u)) {
    case 1: return LC_I16;
    case 2: return LC_I32;
    default: return LC_I64;
  }
}

int norm_axis(int axis, int ndim) {
  int a = axis < 0 ? axis + ndim : axis;
  if (a < 0 || a >= ndim) fail("axis " + std::to_string(axis) + " out of range for rank " + std::to_string(ndim));
  return a;
}

}  // namespace lc

// ------------------------------------------------------------- copy kernels

template <typename CT>
__global__ void k_copy_convert(TV src, char* dst, int dst_dtype, int64_t n) {
  pdl_trigger();
  pdl_wait();
  LC_GRID_STRIDE(i, n) { st_as<CT>(dst, dst_dtype, i, ld_as<CT>(src.ptr, src.dtype, tv_offset(src, i))); }
}

// Same-dtype strided gather in 1/2/4/8-byte units (no conversion).
template <typename U>
__global__ void k_copy_raw(TV src, U* dst, int64_t n) {
  pdl_trigger();
  pdl_wait();
  LC_GRID_STRIDE(i, n) { dst[i] = ((const U*)src.ptr)[tv_offset(src, i)]; }
}

// Same-dtype strided copy whose innermost dimension is dense and spans whole
// 16-byte vectors (every row start 16-byte aligned): one 16-byte load and
// store per thread step, the row offset computed once per vector.
__global__ void k_copy_vec16(TV src, uint4* __restrict__ dst, int64_t nvec, int vpr, int epv) {
  pdl_trigger();
  pdl_wait();
  LC_GRID_STRIDE(i, nvec) {
    int64_t row = i / vpr, off = 0;
    const int c = (int)(i % vpr);
    for (int d = src.ndim - 2; d >= 0; d--) {
      off += (row % src.shape[d]) * src.strides[d];
      row /= src.shape[d];
    }
    dst[i] = *(const uint4*)(src.ptr + (off + (int64_t)c * epv) * (16 / epv));
  }
}

namespace lc {
// Compute type of a dtype conversion a -> b: 0 float, 1 int64, 2 double, 3 uint64.
static int ct_for(int a, int b) {
  if (a == LC_F64 || b == LC_F64) return 2;
  if (a == LC_U64 || b == LC_U64) return 3;
  if (is_float(a)) return is_float(b) ? 0 : 2;  // float -> int truncates through double
  return 1;
}

void copy_into(const LcTensor* src, LcTensor* dst) {
  int64_t n = src->numel();
  if (n == 0) return;
  LC_CHECK(dst->contiguous() && dst->numel() == n, "copy_into: bad destination");
  TV s = tv(src);
  int threads = 256;
  unsigned blocks = blocks_for(n, threads);
  cudaStream_t st = stream();
  if (src->dtype == dst->dtype) {
    if (src->contiguous()) {
      CUDA_OK(cudaMemcpyAsync(dst->data(), src->data(), n * dtype_size(src->dtype), cudaMemcpyDeviceToDevice, st));
      return;
    }
    const int es = (int)dtype_size(src->dtype), epv = 16 / es;
    bool vec = src->ndim >= 1 && es <= 16 && src->strides[src->ndim - 1] == 1 && src->shape[src->ndim - 1] % epv == 0 &&
               (((uintptr_t)src->data() | (uintptr_t)dst->data()) & 15) == 0;
    for (int d = 0; vec && d < src->ndim - 1; d++) vec = (src->strides[d] * es) % 16 == 0;
    if (vec) {
      const int vpr = (int)(src->shape[src->ndim - 1] / epv);
      const int64_t nvec = n / epv;
      lc::launch_chain(k_copy_vec16, dim3(blocks_for(nvec, threads)), dim3(threads), 0, st, s, (uint4*)dst->data(), nvec, vpr, epv);
      LC_LAUNCHED(1);
      return;
    }
    switch (dtype_size(src->dtype)) {
      case 1: lc::launch_chain(k_copy_raw<uint8_t>, dim3(blocks), dim3(threads), 0, st, s, (uint8_t*)dst->data(), n); break;
      case 2: lc::launch_chain(k_copy_raw<uint16_t>, dim3(blocks), dim3(threads), 0, st, s, (uint16_t*)dst->data(), n); break;
      case 4: lc::launch_chain(k_copy_raw<uint32_t>, dim3(blocks), dim3(threads), 0, st, s, (uint32_t*)dst->data(), n); break;
      default: lc::launch_chain(k_copy_raw<uint64_t>, dim3(blocks), dim3(threads), 0, st, s, (uint64_t*)dst->data(), n); break;
    }
  } else {
    // float -> int truncates toward zero; int -> float rounds to nearest.
    int ct = ct_for(src->dtype, dst->dtype);
    switch (ct) {
      case 0: lc::launch_chain(k_copy_convert<float>, dim3(blocks), dim3(threads), 0, st, s, dst->data(), dst->dtype, n); break;
      case 1: lc::launch_chain(k_copy_convert<int64_t>, dim3(blocks), dim3(threads), 0, st, s, dst->data(), dst->dtype, n); break;
      case 2: lc::launch_chain(k_copy_convert<double>, dim3(blocks), dim3(threads), 0, st, s, dst->data(), dst->dtype, n); break;
      default: lc::launch_chain(k_copy_convert<uint64_t>, dim3(blocks), dim3(threads), 0, st, s, dst->data(), dst->dtype, n); break;
    }
  }
  count_launch(1);
  CUDA_OK(cudaGetLastError());
}

LcTensor* contiguous(LcTensor* x) {
  if (x->contiguous()) return x;
  LcTensor* y = alloc(x->dtype, x->dims());
  copy_into(x, y);
  return y;
}

}  // namespace lc

// ------------------------------------------------------------- C ABI

using namespace lc;

extern "C" {

const char* lc_last_error(void) { return g_err.c_str(); }

int lc_init(int device) {
  LC_API_BEGIN
  State& s = S();
  if (s.inited && s.device == device) return 0;
  LC_CHECK(!s.inited, "lc_init: already initialised on another device (one device per process)");
  int n = 0;
  CUDA_OK(cudaGetDeviceCount(&n));
  LC_CHECK(device >= 0 && device < n, "lc_init: no CUDA device " + std::to_string(device));
  CUDA_OK(cudaSetDevice(device));
  cudaDeviceProp prop;
  CUDA_OK(cudaGetDeviceProperties(&prop, device));
  LC_CHECK(prop.major == 10, std::string("lc_init: liblaya_cuda is built for sm_100a (B200); device is ") + prop.name);
  s.sms = prop.multiProcessorCount;
  CUDA_OK(cudaStreamCreateWithFlags(&s.own, cudaStreamNonBlocking));
  s.cur = s.own;
  // keep freed blocks cached in the stream-ordered pool
  cudaMemPool_t pool;
  CUDA_OK(cudaDeviceGetDefaultMemPool(&pool, device));
  uint64_t thr = UINT64_MAX;
  CUDA_OK(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr));
  s.device = device;
  s.inited = true;
  LC_API_END
}

static void destroy_upload_stage();  // the pinned staging of large uploads (lc_from_host)

int lc_destroy(void) {
  LC_API_BEGIN
  State& s = S();
  if (!s.inited) return 0;
  std::vector<LcTensor*> all(s.live.begin(), s.live.end());
  for (auto* t : all) release(t);
  lc_internal_destroy_caches();
  destroy_upload_stage();
  CUDA_OK(cudaStreamSynchronize(s.cur));
  LC_API_END
}

int lc_set_stream(uint64_t stream) {
  LC_API_BEGIN
  ensure_init();
  S().cur = stream ? reinterpret_cast<cudaStream_t>(stream) : S().own;
  LC_API_END
}

int lc_get_stream(uint64_t* out) {
  LC_API_BEGIN
  ensure_init();
  *out = reinterpret_cast<uint64_t>(S().cur);
  LC_API_END
}

int lc_supports(int dtype, int* out) {
  *out = (dtype >= 0 && dtype < LC_NUM_DTYPES) ? 1 : 0;
  return 0;
}

int lc_stats(int64_t* live_tensors, int64_t* live_bytes, int64_t* launches) {
  if (live_tensors) *live_tensors = (int64_t)S().live.size();
  if (live_bytes) *live_bytes = S().live_bytes;
  if (launches) *launches = S().launches;
  return 0;
}

namespace {
// Large uploads go through two pinned staging buffers: the host copies chunk
// i + 1 into one while the DMA engine moves chunk i out of the other (a
// pageable cudaMemcpyAsync runs at a few GB/s; the pinned DMA at tens). Each
// chunk's host copy is split over a few threads. The caller's memory is
// fully read when lc_from_host returns, as fromHost requires; the staging
// buffers are reused only after their DMA has completed (an event per buffer).
constexpr size_t kStageChunk = (size_t)8 << 20;
constexpr size_t kStageMin = (size_t)4 << 20;  // smaller uploads: one pageable copy
struct UploadStage {
  void* buf[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
};
UploadStage& upload_stage() {
  static UploadStage u;
  return u;
}
void host_copy_parallel(void* dst, const void* src, size_t n) {
  const size_t kPart = (size_t)1 << 20;
  const int parts = (int)std::min<size_t>(4, (n + kPart - 1) / kPart);
  if (parts <= 1) {
    std::memcpy(dst, src, n);
    return;
  }
  const size_t per = (n + parts - 1) / parts;
  std::vector<std::thread> ts;
  for (int i = 1; i < parts; i++) {
    const size_t o = per * i, len = std::min(per, n - o);
    ts.emplace_back([=] { std::memcpy((char*)dst + o, (const char*)src + o, len); });
  }
  std::memcpy(dst, src, std::min(per, n));
  for (auto& t : ts) t.join();
}
void upload_staged(void* dev, const void* host, size_t nbytes, cudaStream_t st) {
  UploadStage& u = upload_stage();
  for (int i = 0; i < 2; i++)
    if (!u.buf[i]) {
      CUDA_OK(cudaHostAlloc(&u.buf[i], kStageChunk, cudaHostAllocDefault));
      CUDA_OK(cudaEventCreateWithFlags(&u.done[i], cudaEventDisableTiming));
      CUDA_OK(cudaEventRecord(u.done[i], st));
    }
  int k = 0;
  for (size_t o = 0; o < nbytes; o += kStageChunk, k ^= 1) {
    const size_t len = std::min(kStageChunk, nbytes - o);
    CUDA_OK(cudaEventSynchronize(u.done[k]));  // the previous DMA out of this buffer has finished
    host_copy_parallel(u.buf[k], (const char*)host + o, len);
    CUDA_OK(cudaMemcpyAsync((char*)dev + o, u.buf[k], len, cudaMemcpyHostToDevice, st));
    CUDA_OK(cudaEventRecord(u.done[k], st));
  }
}
}  // namespace

static void destroy_upload_stage() {
  UploadStage& u = upload_stage();
  for (int i = 0; i < 2; i++) {
    if (u.done[i]) cudaEventSynchronize(u.done[i]), cudaEventDestroy(u.done[i]);
    if (u.buf[i]) cudaFreeHost(u.buf[i]);
    u.buf[i] = nullptr;
    u.done[i] = nullptr;
  }
}

int lc_from_host(lc_tensor* out, int dtype, const int64_t* shape, int ndim, const void* data, size_t nbytes) {
  LC_API_BEGIN
  LC_CHECK(dtype >= 0 && dtype < LC_NUM_DTYPES, "fromHost: unknown dtype");
  LC_CHECK(ndim >= 0 && ndim <= LC_MAX_DIMS, "fromHost: rank must be 0..8");
  std::vector<int64_t> sh(shape, shape + ndim);
  int64_t n = 1;
  for (auto d : sh) n *= d;
  LC_CHECK((size_t)n * dtype_size(dtype) == nbytes,
           "fromHost: " + std::to_string(nbytes) + " bytes for " + dtype_name(dtype) + " " + shape_str(sh));
  LcTensor* t = alloc(dtype, sh);
  if (nbytes) {
    // pageable source: the copy is complete (staged) when cudaMemcpyAsync returns,
    // so the caller may reuse `data` at once (index.ts:146-154). While a graph is
    // captured the copy is the capture's (no host-side staging).
    if (nbytes >= kStageMin && !S().capturing) upload_staged(t->data(), data, nbytes, stream());
    else CUDA_OK(cudaMemcpyAsync(t->data(), data, nbytes, cudaMemcpyHostToDevice, stream()));
  }
  t->st->upload_mark = S().launches;
  *out = handle(t);
  LC_API_END
}

int lc_from_device(lc_tensor* out, int dtype, const int64_t* shape, int ndim, void* dptr) {
  LC_API_BEGIN
  LC_CHECK(dtype >= 0 && dtype < LC_NUM_DTYPES, "fromDevice: unknown dtype");
  LC_CHECK(ndim >= 0 && ndim <= LC_MAX_DIMS, "fromDevice: rank must be 0..8");
  std::vector<int64_t> sh(shape, shape + ndim);
  LcStorage* st = new LcStorage();
  st->ptr = dptr;
  st->external = true;
  int64_t n = 1;
  for (auto d : sh) n *= d;
  st->bytes = n * dtype_size(dtype);
  *out = handle(new_tensor(st, dtype, sh));
  LC_API_END
}

int lc_read(lc_tensor h, void* dst, size_t nbytes) {
  LC_API_BEGIN
  LcTensor* t = check(h, "read");
  size_t want = (size_t)t->numel() * dtype_size(t->dtype);
  LC_CHECK(want == nbytes, "read: buffer has " + std::to_string(nbytes) + " bytes, tensor needs " + std::to_string(want));
  LcTensor* c = contiguous(t);
  if (nbytes) CUDA_OK(cudaMemcpyAsync(dst, c->data(), nbytes, cudaMemcpyDeviceToHost, stream()));
  CUDA_OK(cudaStreamSynchronize(stream()));
  if (c != t) release(c);
  LC_API_END
}

int lc_tensor_free(lc_tensor h) {
  LC_API_BEGIN
  LcTensor* t = check(h, "dispose");
  release(t);
  LC_API_END
}

int lc_tensor_info(lc_tensor h, int* dtype, int* ndim, int64_t* shape) {
  LC_API_BEGIN
  LcTensor* t = check(h, "info");
  *dtype = t->dtype;
  *ndim = t->ndim;
  for (int i = 0; i < t->ndim; i++) shape[i] = t->shape[i];
  LC_API_END
}

int lc_tensor_data(lc_tensor h, uint64_t* dptr) {
  LC_API_BEGIN
  LcTensor* t = check(h, "data");
  *dptr = t->contiguous() ? reinterpret_cast<uint64_t>(t->data()) : 0;
  LC_API_END
}

int lc_flush(void) {
  LC_API_BEGIN
  ensure_init();
  CUDA_OK(cudaStreamSynchronize(stream()));
  std::string err = take_device_errors();
  LC_CHECK(err.empty(), err);
  LC_API_END
}

int lc_reshape(lc_tensor* out, lc_tensor xh, const int64_t* shape, int ndim) {
  LC_API_BEGIN
  LcTensor* x = check(xh, "reshape");
  LC_CHECK(ndim >= 0 && ndim <= LC_MAX_DIMS, "reshape: rank must be 0..8");
  std::vector<int64_t> sh(shape, shape + ndim);
  int64_t n = x->numel(), known = 1;
  int infer = -1;
  for (int i = 0; i < ndim; i++) {
    if (sh[i] == -1) {
      LC_CHECK(infer < 0, "reshape: more than one -1");
      infer = i;
    } else {
      LC_CHECK(sh[i] >= 0, "reshape: negative dimension");
      known *= sh[i];
    }
  }
  if (infer >= 0) {
    LC_CHECK(known > 0 && n % known == 0, "reshape: cannot infer -1 for " + shape_str(x->dims()));
    sh[infer] = n / known;
    known *= sh[infer];
  }
  LC_CHECK(known == n, "reshape: " + shape_str(x->dims()) + " -> " + shape_str(sh) + " changes the size");
  // A view when the old strides allow it (numpy's no-copy reshape rule): drop
  // size-1 axes, then match groups of old and new axes with equal products;
  // each old group must be internally contiguous.
  {
    std::vector<int64_t> od, os;
    for (int i = 0; i < x->ndim; i++)
      if (x->shape[i] != 1) od.push_back(x->shape[i]), os.push_back(x->strides[i]);
    std::vector<int64_t> nst(ndim, 0);
    bool ok = n > 0;
    size_t oi = 0;
    int ni = 0;
    while (ok && ni < ndim) {
      if (sh[ni] == 1) {
        nst[ni] = 1;
        ni++;
        continue;
      }
      if (oi >= od.size()) { ok = false; break; }
      int64_t np_ = sh[ni], op_ = od[oi];
      int nj = ni;
      size_t oj = oi;
      while (np_ != op_) {
        if (np_ < op_) { if (++nj >= ndim) { ok = false; break; } np_ *= sh[nj]; }
        else { if (++oj >= od.size()) { ok = false; break; } op_ *= od[oj]; }
      }
      if (!ok) break;
      for (size_t k = oi; k < oj; k++)
        if (os[k] != os[k + 1] * od[k + 1]) ok = false;
      if (!ok) break;
      int64_t st = os[oj];
      for (int k = nj; k >= ni; k--) {
        nst[k] = st;
        st *= sh[k];
      }
      ni = nj + 1;
      oi = oj + 1;
    }
    if (ok && oi == od.size()) {
      *out = handle(view_of(x, sh, nst, x->offset));
      return 0;
    }
  }
  LcTensor* src = contiguous(x);
  std::vector<int64_t> st(ndim);
  int64_t s = 1;
  for (int i = ndim - 1; i >= 0; i--) {
    st[i] = s;
    s *= sh[i];
  }
  LcTensor* y = view_of(src, sh, st, src->offset);
  if (src != x) release(src);
  *out = handle(y);
  LC_API_END
}

int lc_transpose(lc_tensor* out, lc_tensor xh, const int32_t* perm, int ndim) {
  LC_API_BEGIN
  LcTensor* x = check(xh, "transpose");
  LC_CHECK(ndim == x->ndim, "transpose: perm length differs from rank");
  std::vector<int64_t> sh(ndim), st(ndim);
  std::vector<bool> seen(ndim, false);
  for (int i = 0; i < ndim; i++) {
    int p = norm_axis(perm[i], ndim);
    LC_CHECK(!seen[p], "transpose: repeated axis");
    seen[p] = true;
    sh[i] = x->shape[p];
    st[i] = x->strides[p];
  }
  *out = handle(view_of(x, sh, st, x->offset));
  LC_API_END
}

int lc_slice(lc_tensor* out, lc_tensor xh, const int64_t* begin, const int64_t* end, int n) {
  LC_API_BEGIN
  LcTensor* x = check(xh, "slice");
  LC_CHECK(n <= x->ndim, "slice: more bounds than axes");
  std::vector<int64_t> sh = x->dims(), st(x->strides, x->strides + x->ndim);
  int64_t off = x->offset;
  for (int i = 0; i < n; i++) {
    int64_t d = x->shape[i];
    int64_t b = begin[i] < 0 ? begin[i] + d : begin[i];
    int64_t e = end[i] < 0 ? end[i] + d : end[i];
    b = std::max<int64_t>(0, std::min(b, d));
    e = std::max<int64_t>(b, std::min(e, d));
    sh[i] = e - b;
    off += b * x->strides[i];
  }
  *out = handle(view_of(x, sh, st, off));
  LC_API_END
}

int lc_split(lc_tensor* outs, lc_tensor xh, int parts, int axis) {
  LC_API_BEGIN
  LcTensor* x = check(xh, "split");
  int a = norm_axis(axis, x->ndim);
  LC_CHECK(parts > 0 && x->shape[a] % parts == 0, "split: axis of size " + std::to_string(x->shape[a]) + " is not divisible into " + std::to_string(parts));
  int64_t w = x->shape[a] / parts;
  std::vector<int64_t> sh = x->dims(), st(x->strides, x->strides + x->ndim);
  sh[a] = w;
  for (int p = 0; p < parts; p++) outs[p] = handle(view_of(x, sh, st, x->offset + p * w * x->strides[a]));
  LC_API_END
}

int lc_concat(lc_tensor* out, const lc_tensor* xs, int n, int axis) {
  LC_API_BEGIN
  LC_CHECK(n > 0, "concat: no inputs");
  std::vector<LcTensor*> ts;
  for (int i = 0; i < n; i++) ts.push_back(check(xs[i], "concat"));
  int r = ts[0]->ndim;
  int a = norm_axis(axis, r);
  int dt = ts[0]->dtype;
  std::vector<int64_t> sh = ts[0]->dims();
  sh[a] = 0;
  for (auto* t : ts) {
    LC_CHECK(t->ndim == r, "concat: rank mismatch");
    for (int i = 0; i < r; i++)
      if (i != a) LC_CHECK(t->shape[i] == ts[0]->shape[i], "concat: shape mismatch off the concat axis");
    sh[a] += t->shape[a];
    dt = promote(dt, t->dtype);
  }
  LcTensor* y = alloc(dt, sh);
  // copy each piece into the strided window of y
  int64_t at = 0;
  for (auto* t : ts) {
    if (t->numel() == 0) {
      at += t->shape[a];
      continue;
    }
    std::vector<int64_t> st(y->strides, y->strides + r);
    LcTensor* win = view_of(y, t->dims(), st, at * y->strides[a]);
    // strided destination: write through a converting scatter
    lc_internal_copy_strided(t, win);
    release(win);
    at += t->shape[a];
  }
  *out = handle(y);
  LC_API_END
}

int lc_cast(lc_tensor* out, lc_tensor xh, int dtype) {
  LC_API_BEGIN
  LcTensor* x = check(xh, "cast");
  LC_CHECK(dtype >= 0 && dtype < LC_NUM_DTYPES, "cast: unknown dtype");
  LcTensor* y = alloc(dtype, x->dims());
  copy_into(x, y);
  *out = handle(y);
  LC_API_END
}

}  // extern "C"

// ------------------------------------------------------------- captured graphs (Backend.compile)
//
// The op sequence issued between lc_graph_capture_begin and _end is recorded
// from the library stream into a CUDA graph and replayed by lc_graph_launch
// on the same tensors' memory. Memory the captured ops allocate is the
// graph's (stream-ordered alloc/free nodes); whatever a replay must hand
// back has to be copied out to memory that existed before the capture
// (lc_copy_into) and the captured tensors disposed before _end.

namespace {
constexpr uint64_t kGraphMagic = 0x4c43475241504831ull;
struct LcGraph {
  uint64_t magic = kGraphMagic;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  std::vector<void*> deferred;  // freed with the graph
};
std::unordered_set<LcGraph*>& graphs() {
  static std::unordered_set<LcGraph*> g;
  return g;
}
void end_capture_state(std::vector<void*>* keep) {
  State& s = S();
  s.capturing = false;
  s.cap_allocs.clear();
  if (keep) keep->swap(s.cap_deferred);
  for (void* p : s.cap_deferred) cudaFreeAsync(p, s.cur);
  s.cap_deferred.clear();
}
LcGraph* check_graph(uint64_t h) {
  LcGraph* g = reinterpret_cast<LcGraph*>(h);
  LC_CHECK(h && graphs().count(g) && g->magic == kGraphMagic, "graph: not a live graph handle");
  return g;
}
}  // namespace

extern "C" {

int lc_graph_capture_begin(void) {
  LC_API_BEGIN
  ensure_init();
  State& s = S();
  LC_CHECK(!s.capturing, "graph capture: a capture is already in progress");
  CUDA_OK(cudaStreamBeginCapture(s.cur, cudaStreamCaptureModeRelaxed));
  s.capturing = true;
  LC_API_END
}

int lc_graph_capture_end(uint64_t* out) {
  LC_API_BEGIN
  ensure_init();
  State& s = S();
  LC_CHECK(s.capturing, "graph capture: no capture in progress");
  capture_ending(false);
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(s.cur, &graph);
  const size_t unfreed = s.cap_allocs.size();
  auto g = std::make_unique<LcGraph>();
  end_capture_state(&g->deferred);
  if (e != cudaSuccess || !graph || unfreed) {
    cudaGetLastError();
    if (graph) cudaGraphDestroy(graph);
    for (void* p : g->deferred) cudaFreeAsync(p, s.cur);
    if (e != cudaSuccess || !graph)
      fail(std::string("graph capture failed: ") + cudaGetErrorString(e) +
           " (an op synchronised with the host or used another stream while capturing)");
    fail("graph capture: " + std::to_string(unfreed) + " allocations made while capturing were not released before the end");
  }
  g->graph = graph;
  e = cudaGraphInstantiateWithFlags(&g->exec, graph, 0);
  if (e != cudaSuccess) {
    cudaGetLastError();
    cudaGraphDestroy(graph);
    for (void* p : g->deferred) cudaFreeAsync(p, s.cur);
    fail(std::string("graph instantiate failed: ") + cudaGetErrorString(e));
  }
  LcGraph* raw = g.release();
  graphs().insert(raw);
  *out = reinterpret_cast<uint64_t>(raw);
  LC_API_END
}

int lc_graph_capture_abort(void) {
  LC_API_BEGIN
  ensure_init();
  State& s = S();
  if (!s.capturing) return 0;
  cudaGraph_t graph = nullptr;
  cudaStreamEndCapture(s.cur, &graph);
  cudaGetLastError();
  if (graph) cudaGraphDestroy(graph);
  capture_ending(true);
  end_capture_state(nullptr);
  LC_API_END
}

int lc_graph_launch(uint64_t h) {
  LC_API_BEGIN
  ensure_init();
  LcGraph* g = check_graph(h);
  LC_CHECK(!S().capturing, "graph launch: not allowed while capturing");
  CUDA_OK(cudaGraphLaunch(g->exec, S().cur));
  S().launches += 1;
  LC_API_END
}

int lc_graph_destroy(uint64_t h) {
  LC_API_BEGIN
  ensure_init();
  LcGraph* g = check_graph(h);
  graphs().erase(g);
  // launches already queued on the stream finish before the stream-ordered frees
  if (g->exec) cudaGraphExecDestroy(g->exec);
  if (g->graph) cudaGraphDestroy(g->graph);
  for (void* p : g->deferred) cudaFreeAsync(p, S().cur);
  g->magic = 0;
  delete g;
  LC_API_END
}

int lc_copy_into(lc_tensor dsth, lc_tensor srch) {
  LC_API_BEGIN
  LcTensor* dst = check(dsth, "copyInto dst");
  LcTensor* src = check(srch, "copyInto src");
  LC_CHECK(dst->dtype == src->dtype && dst->dims() == src->dims(),
           "copyInto: dst " + std::string(dtype_name(dst->dtype)) + shape_str(dst->dims()) + " vs src " + dtype_name(src->dtype) +
               shape_str(src->dims()));
  LC_CHECK(dst->contiguous(), "copyInto: the destination must be dense");
  dst->st->upload_mark = -1;
  dst->st->version++;
  copy_into(src, dst);
  LC_API_END
}

}  // extern "C"

// ------------------------------------------------------------- failure-path test hooks
void lc_internal_wait_limit_gemm(unsigned long long ns);
void lc_internal_wait_limit_attention(unsigned long long ns);
void lc_internal_wait_limit_encoder(unsigned long long ns);
void lc_internal_launch_wait_probe();

extern "C" {

int lc_debug_set_wait_limit(uint64_t ns) {
  LC_API_BEGIN
  ensure_init();
  const unsigned long long v = ns ? (unsigned long long)ns : 2000000000ull;
  lc_internal_wait_limit_gemm(v);
  lc_internal_wait_limit_attention(v);
  lc_internal_wait_limit_encoder(v);
  LC_API_END
}

int lc_debug_set_alloc_cap(int64_t bytes) {
  LC_API_BEGIN
  ensure_init();
  LC_CHECK(bytes >= 0, "allocation cap must be >= 0");
  S().alloc_cap = bytes;
  LC_API_END
}

int lc_debug_stuck_wait(void) {
  LC_API_BEGIN
  ensure_init();
  lc_internal_launch_wait_probe();
  LC_API_END
}

}  // extern "C"
