// Flash attention over unpadded variable-length sequences, head dim 64:
// the attention of the ModernBERT encoder layer (packages/modernbert/src/index.ts:348-352,
// the contract's `sdpa` with the masks of attentionMasks, index.ts:240-259)
// without materialising masks or padding.
//
// Input  qkv [T, 3·H] (the fused Wqkv projection, RoPE already applied by the
//        GEMM epilogue): q of head h at columns h·64, k at H + h·64, v at 2H + h·64.
// Output att [T, H] (head h at columns h·64), the layout the Wo GEMM reads.
// Global layers see every key of their own sequence; sliding layers see keys
// with |i − j| ≤ window/2, so a 64-row query tile touches at most 3 key tiles.
//
// One CTA = 64 query rows x one head, 4 warps x 16 rows. Q·Kᵀ and P·V run on
// mma.sync m16n8k16 (f16/bf16 in, f32 accumulate) with ldmatrix from a
// 128-byte-XOR-swizzled shared-memory tile; K/V tiles are double-buffered with
// cp.async; the softmax is the online (running max / sum) form in f32, base 2.
#include "lc_api.h"
#include "lc_gemm.h"

namespace {

constexpr int HD = 64;      // head dim
constexpr int QT = 64;      // query rows per CTA
constexpr int KT = 64;      // keys per tile

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// element offset (in halves) of (row, chunk of 8) in a swizzled [64][64] tile
__device__ __forceinline__ int swz(int row, int chunk) { return row * HD + ((chunk ^ (row & 7)) << 3); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldm_x4(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldm_x4_t(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

template <typename T> struct Mma;
template <> struct Mma<__half> {
  __device__ static void run(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ static uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *(uint32_t*)&h;
  }
};
template <> struct Mma<__nv_bfloat16> {
  __device__ static void run(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ static uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *(uint32_t*)&h;
  }
};

struct AttnArgs {
  const void* qkv;
  void* out;
  const int4* tiles;  // (first token of the sequence, its length, first query row of the tile, 0)
  int64_t T;          // total tokens (rows of qkv)
  int H;              // hidden size = heads * 64
  int half_window;    // sliding: keys with |i - j| <= half_window; < 0 = global
  float scale_log2;   // softmax scale * log2(e)
};

// copy rows [r0, r0+64) x 64 columns starting at `col` of the [T, 3H] qkv matrix into a swizzled tile
template <typename T>
__device__ __forceinline__ void load_tile(T* s, const T* qkv, int64_t tok0, int r0, int len, int64_t ld, int col, int64_t Tn) {
#pragma unroll
  for (int i = 0; i < (64 * 8) / 128; i++) {
    int idx = threadIdx.x + i * 128;
    int row = idx >> 3, ch = idx & 7;
    int r = r0 + row;
    int64_t tok = tok0 + (r < len ? r : len - 1);  // clamp inside the sequence (masked later)
    if (tok >= Tn) tok = Tn - 1;
    cp_async16(s + swz(row, ch), qkv + tok * ld + col + ch * 8);
  }
}

template <typename T, bool LOCAL>
__global__ void __launch_bounds__(128) k_flash_varlen(const AttnArgs a) {
  __shared__ __align__(128) T sQ[QT * HD];
  __shared__ __align__(128) T sK[2][KT * HD];
  __shared__ __align__(128) T sV[2][KT * HD];
  const int4 tile = a.tiles[blockIdx.x];
  const int64_t tok0 = tile.x;
  const int L = tile.y, q0 = tile.z;
  const int h = blockIdx.y;
  const int64_t ld = 3 * (int64_t)a.H;
  const T* qkv = (const T*)a.qkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;

  int kv_lo = 0, kv_hi = L;
  if (LOCAL) {
    kv_lo = max(0, q0 - a.half_window);
    kv_hi = min(L, q0 + QT - 1 + a.half_window + 1);
  }
  kv_lo = (kv_lo / KT) * KT;
  const int ntiles = (kv_hi - kv_lo + KT - 1) / KT;

  load_tile<T>(sQ, qkv, tok0, q0, L, ld, h * HD, a.T);
  load_tile<T>(sK[0], qkv, tok0, kv_lo, L, ld, a.H + h * HD, a.T);
  load_tile<T>(sV[0], qkv, tok0, kv_lo, L, ld, 2 * a.H + h * HD, a.T);
  cp_commit();

  float o[8][4];
#pragma unroll
  for (int j = 0; j < 8; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  uint32_t qa[4][4];
  const int qrow0 = q0 + warp * 16 + g;  // this thread's two query rows: qrow0, qrow0 + 8

  for (int it = 0; it < ntiles; it++) {
    const int buf = it & 1;
    if (it + 1 < ntiles) {
      const int kn = kv_lo + (it + 1) * KT;
      load_tile<T>(sK[buf ^ 1], qkv, tok0, kn, L, ld, a.H + h * HD, a.T);
      load_tile<T>(sV[buf ^ 1], qkv, tok0, kn, L, ld, 2 * a.H + h * HD, a.T);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (it == 0) {
      // Q fragments for the 4 k-steps of this warp's 16 rows
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        int row = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        int ch = kk * 2 + (lane >> 4);
        ldm_x4(qa[kk], sQ + swz(row, ch));
      }
    }
    const T* K = sK[buf];
    const T* V = sV[buf];
    // S = Q Kᵀ : 16 x 64 per warp = 8 n-tiles of 8 keys
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
#pragma unroll
      for (int jp = 0; jp < 4; jp++) {  // pairs of n-tiles (16 keys)
        uint32_t b[4];
        int key = jp * 16 + (lane & 7) + (lane >> 4) * 8;
        int ch = kk * 2 + ((lane >> 3) & 1);
        ldm_x4(b, K + swz(key, ch));
        Mma<T>::run(s[2 * jp], qa[kk], b[0], b[1]);
        Mma<T>::run(s[2 * jp + 1], qa[kk], b[2], b[3]);
      }
    }
    // scale, mask, online softmax
    const int kbase = kv_lo + it * KT;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; j++) {
#pragma unroll
      for (int e = 0; e < 4; e++) {
        int key = kbase + j * 8 + 2 * t4 + (e & 1);
        int qi = qrow0 + ((e >> 1) << 3);
        bool ok = key < L;
        if (LOCAL) ok = ok && (key - qi <= a.half_window) && (qi - key <= a.half_window);
        float v = ok ? s[j][e] * a.scale_log2 : -INFINITY;
        s[j][e] = v;
        if (e < 2) mx0 = fmaxf(mx0, v);
        else mx1 = fmaxf(mx1, v);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float b0 = n0 == -INFINITY ? 0.f : n0, b1 = n1 == -INFINITY ? 0.f : n1;
    const float c0 = exp2f(m0 - b0), c1 = exp2f(m1 - b1);
    m0 = n0;
    m1 = n1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      s[j][0] = exp2f(s[j][0] - b0);
      s[j][1] = exp2f(s[j][1] - b0);
      s[j][2] = exp2f(s[j][2] - b1);
      s[j][3] = exp2f(s[j][3] - b1);
      rs0 += s[j][0] + s[j][1];
      rs1 += s[j][2] + s[j][3];
    }
    l0 = l0 * c0 + rs0;
    l1 = l1 * c1 + rs1;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      o[j][0] *= c0;
      o[j][1] *= c0;
      o[j][2] *= c1;
      o[j][3] *= c1;
    }
    // O += P V : P (16 x 64 keys) as A fragments, V via ldmatrix.trans
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      uint32_t pa[4];
      pa[0] = Mma<T>::pack(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = Mma<T>::pack(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = Mma<T>::pack(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = Mma<T>::pack(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < 4; dp++) {  // pairs of 8-dim n-tiles
        uint32_t b[4];
        int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        int ch = dp * 2 + (lane >> 4);
        ldm_x4_t(b, V + swz(key, ch));
        Mma<T>::run(o[2 * dp], pa, b[0], b[1]);
        Mma<T>::run(o[2 * dp + 1], pa, b[2], b[3]);
      }
    }
    __syncthreads();  // the buffer is refilled next iteration
  }
  // finish: row sums across the quad, normalise, store
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float i0 = 1.f / l0, i1 = 1.f / l1;
  T* out = (T*)a.out;
  const int r0 = qrow0, r1 = qrow0 + 8;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    int col = h * HD + j * 8 + 2 * t4;
    if (r0 < L) *(uint32_t*)(out + (tok0 + r0) * a.H + col) = Mma<T>::pack(o[j][0] * i0, o[j][1] * i0);
    if (r1 < L) *(uint32_t*)(out + (tok0 + r1) * a.H + col) = Mma<T>::pack(o[j][2] * i1, o[j][3] * i1);
  }
}

// ---- the contract's sdpa (index.ts:230-237) on tensor cores: softmax(q·kᵀ·scale
// masked by a bool mask)·v with q [B, H, Lq, 64], k / v [B, H, Lk, 64] given by
// strides (last dimension dense, rows 16-byte aligned: the views ModernBert.layer
// makes with reshape / transpose / split, packages/modernbert/src/index.ts:342-352),
// mask any bool tensor broadcast to [B, H, Lq, Lk] (the attentionMasks
// [B, 1, 1, L] / [B, 1, L, L] of index.ts:240-259) or none. Same tiles and
// online softmax as k_flash_varlen: one CTA = 64 query rows of one (b, h).
// A fully masked row gets 0/0, as the generic kernel (the contract leaves it
// undefined).
struct SdpaArgs {
  const void* q;
  const void* k;
  const void* v;
  const uint8_t* m;     // null: no mask
  int64_t qs[3], ks[3], vs[3];  // element strides of batch, head, row
  int64_t ms[4];        // mask strides of batch, head, query, key (0 where broadcast)
  int H, Lq, Lk;
  float scale_log2;     // scale * log2(e)
  void* y;              // [B, H, Lq, 64] dense
};

// rows [r0, r0+64) of a [len, 64] strided matrix into a swizzled tile (rows past
// the end repeat the last row; their scores are masked)
template <typename T>
__device__ __forceinline__ void load_rows(T* s, const T* base, int r0, int len, int64_t ld) {
#pragma unroll
  for (int i = 0; i < (64 * 8) / 128; i++) {
    const int idx = threadIdx.x + i * 128;
    const int row = idx >> 3, ch = idx & 7;
    const int r = min(r0 + row, len - 1);
    cp_async16(s + swz(row, ch), base + (int64_t)r * ld + ch * 8);
  }
}

template <typename T>
__global__ void __launch_bounds__(128) k_sdpa_flash(const SdpaArgs a) {
  __shared__ __align__(128) T sQ[QT * HD];
  __shared__ __align__(128) T sK[2][KT * HD];
  __shared__ __align__(128) T sV[2][KT * HD];
  const int q0 = blockIdx.x * QT;
  const int bh = blockIdx.y, bi = bh / a.H, h = bh % a.H;
  const T* Q = (const T*)a.q + bi * a.qs[0] + h * a.qs[1];
  const T* Kp = (const T*)a.k + bi * a.ks[0] + h * a.ks[1];
  const T* Vp = (const T*)a.v + bi * a.vs[0] + h * a.vs[1];
  const uint8_t* Mk = a.m ? a.m + bi * a.ms[0] + h * a.ms[1] : nullptr;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int ntiles = (a.Lk + KT - 1) / KT;

  load_rows<T>(sQ, Q, q0, a.Lq, a.qs[2]);
  load_rows<T>(sK[0], Kp, 0, a.Lk, a.ks[2]);
  load_rows<T>(sV[0], Vp, 0, a.Lk, a.vs[2]);
  cp_commit();

  float o[8][4];
#pragma unroll
  for (int j = 0; j < 8; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  uint32_t qa[4][4];
  const int qrow0 = q0 + warp * 16 + g;  // this thread's two query rows: qrow0, qrow0 + 8
  const uint8_t* mrow0 = Mk ? Mk + (int64_t)min(qrow0, a.Lq - 1) * a.ms[2] : nullptr;
  const uint8_t* mrow1 = Mk ? Mk + (int64_t)min(qrow0 + 8, a.Lq - 1) * a.ms[2] : nullptr;

  for (int it = 0; it < ntiles; it++) {
    const int buf = it & 1;
    if (it + 1 < ntiles) {
      load_rows<T>(sK[buf ^ 1], Kp, (it + 1) * KT, a.Lk, a.ks[2]);
      load_rows<T>(sV[buf ^ 1], Vp, (it + 1) * KT, a.Lk, a.vs[2]);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (it == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        int row = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        int ch = kk * 2 + (lane >> 4);
        ldm_x4(qa[kk], sQ + swz(row, ch));
      }
    }
    const T* K = sK[buf];
    const T* V = sV[buf];
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
#pragma unroll
      for (int jp = 0; jp < 4; jp++) {
        uint32_t b[4];
        int key = jp * 16 + (lane & 7) + (lane >> 4) * 8;
        int ch = kk * 2 + ((lane >> 3) & 1);
        ldm_x4(b, K + swz(key, ch));
        Mma<T>::run(s[2 * jp], qa[kk], b[0], b[1]);
        Mma<T>::run(s[2 * jp + 1], qa[kk], b[2], b[3]);
      }
    }
    const int kbase = it * KT;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; j++) {
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int key = kbase + j * 8 + 2 * t4 + (e & 1);
        bool ok = key < a.Lk;
        if (ok && Mk) ok = ((e >> 1) ? mrow1 : mrow0)[(int64_t)key * a.ms[3]] != 0;
        const float v = ok ? s[j][e] * a.scale_log2 : -INFINITY;
        s[j][e] = v;
        if (e < 2) mx0 = fmaxf(mx0, v);
        else mx1 = fmaxf(mx1, v);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float b0 = n0 == -INFINITY ? 0.f : n0, b1 = n1 == -INFINITY ? 0.f : n1;
    const float c0 = exp2f(m0 - b0), c1 = exp2f(m1 - b1);
    m0 = n0;
    m1 = n1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      s[j][0] = exp2f(s[j][0] - b0);
      s[j][1] = exp2f(s[j][1] - b0);
      s[j][2] = exp2f(s[j][2] - b1);
      s[j][3] = exp2f(s[j][3] - b1);
      rs0 += s[j][0] + s[j][1];
      rs1 += s[j][2] + s[j][3];
    }
    l0 = l0 * c0 + rs0;
    l1 = l1 * c1 + rs1;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      o[j][0] *= c0;
      o[j][1] *= c0;
      o[j][2] *= c1;
      o[j][3] *= c1;
    }
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      uint32_t pa[4];
      pa[0] = Mma<T>::pack(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = Mma<T>::pack(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = Mma<T>::pack(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = Mma<T>::pack(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < 4; dp++) {
        uint32_t b[4];
        int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        int ch = dp * 2 + (lane >> 4);
        ldm_x4_t(b, V + swz(key, ch));
        Mma<T>::run(o[2 * dp], pa, b[0], b[1]);
        Mma<T>::run(o[2 * dp + 1], pa, b[2], b[3]);
      }
    }
    __syncthreads();
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float i0 = 1.f / l0, i1 = 1.f / l1;
  T* out = (T*)a.y + (int64_t)bh * a.Lq * HD;
  const int r0 = qrow0, r1 = qrow0 + 8;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int col = j * 8 + 2 * t4;
    if (r0 < a.Lq) *(uint32_t*)(out + (int64_t)r0 * HD + col) = Mma<T>::pack(o[j][0] * i0, o[j][1] * i0);
    if (r1 < a.Lq) *(uint32_t*)(out + (int64_t)r1 * HD + col) = Mma<T>::pack(o[j][2] * i1, o[j][3] * i1);
  }
}

}  // namespace

namespace lc {

// The contract's sdpa on tensor cores when the operands allow it (f16/bf16,
// head dim 64, dense rows 16-byte aligned, y dense in q's dtype); false
// (nothing launched) otherwise.
bool sdpa_flash(const LcTensor* q, const LcTensor* k, const LcTensor* v, const LcTensor* m, float scale, LcTensor* y) {
  if (!is_half(q->dtype) || k->dtype != q->dtype || v->dtype != q->dtype || y->dtype != q->dtype || !y->contiguous()) return false;
  const int64_t B = q->shape[0], H = q->shape[1], Lq = q->shape[2], Lk = k->shape[2];
  if (q->shape[3] != HD || v->shape[3] != HD || Lq < 1 || Lk < 1 || B * H > 65535 || Lq > INT32_MAX || Lk > INT32_MAX) return false;
  for (const LcTensor* t : {q, k, v}) {
    if (t->strides[3] != 1 || ((uintptr_t)t->data() & 15)) return false;
    for (int d = 0; d < 3; d++)
      if (t->shape[d] > 1 && t->strides[d] % 8) return false;  // a size-1 axis's stride is never used
  }
  SdpaArgs a{};
  a.q = q->data();
  a.k = k->data();
  a.v = v->data();
  for (int i = 0; i < 3; i++) {
    a.qs[i] = q->strides[i];
    a.ks[i] = k->strides[i];
    a.vs[i] = v->strides[i];
  }
  if (m) {
    TV mv = tv_broadcast(m, {B, H, Lq, Lk});
    a.m = (const uint8_t*)mv.ptr;
    for (int i = 0; i < 4; i++) a.ms[i] = mv.strides[i];
  }
  a.H = (int)H;
  a.Lq = (int)Lq;
  a.Lk = (int)Lk;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.y = y->data();
  dim3 grid((unsigned)((Lq + QT - 1) / QT), (unsigned)(B * H));
  if (q->dtype == LC_F16) k_sdpa_flash<__half><<<grid, 128, 0, stream()>>>(a);
  else k_sdpa_flash<__nv_bfloat16><<<grid, 128, 0, stream()>>>(a);
  LC_LAUNCHED(1);
  return true;
}

// Tile list for cu_seqlens (host): one entry per 64-row query tile of each sequence.
std::vector<int4> attention_tiles(const int32_t* cu, int nseq) {
  std::vector<int4> t;
  for (int s = 0; s < nseq; s++) {
    int L = cu[s + 1] - cu[s];
    for (int q0 = 0; q0 < L; q0 += QT) t.push_back(make_int4(cu[s], L, q0, 0));
  }
  return t;
}

void attention_varlen(const void* qkv, void* out, const int4* tiles_dev, int ntiles, int64_t T, int H, int half_window, float scale,
                      int dtype, cudaStream_t st) {
  LC_CHECK(H % HD == 0, "attention: head dim must be 64");
  if (ntiles == 0) return;
  AttnArgs a{qkv, out, tiles_dev, T, H, half_window, scale * 1.4426950408889634f};
  dim3 grid((unsigned)ntiles, (unsigned)(H / HD));
  LC_CHECK(ntiles < (1 << 30), "attention: too many tiles");
  if (dtype == LC_F16) {
    if (half_window >= 0) k_flash_varlen<__half, true><<<grid, 128, 0, st>>>(a);
    else k_flash_varlen<__half, false><<<grid, 128, 0, st>>>(a);
  } else {
    if (half_window >= 0) k_flash_varlen<__nv_bfloat16, true><<<grid, 128, 0, st>>>(a);
    else k_flash_varlen<__nv_bfloat16, false><<<grid, 128, 0, st>>>(a);
  }
  LC_LAUNCHED(1);
}

}  // namespace lc

using namespace lc;

extern "C" int lc_attention_varlen(lc_tensor* out, lc_tensor qkvh, const int32_t* cu_seqlens, int nseq, int half_window, double scale,
                                   int kernel) {
  LC_API_BEGIN
  LC_CHECK(kernel == 0 || kernel == 1, "attentionVarlen: kernel must be 0 (tcgen05) or 1 (mma.sync)");
  LcTensor* qkv = check(qkvh, "attentionVarlen qkv");
  LC_CHECK(qkv->ndim == 2 && qkv->contiguous() && is_half(qkv->dtype), "attentionVarlen: qkv must be a dense f16/bf16 [T, 3H] matrix");
  LC_CHECK(qkv->shape[1] % (3 * HD) == 0, "attentionVarlen: qkv columns must be 3 x heads x 64");
  int64_t T = qkv->shape[0];
  int H = (int)(qkv->shape[1] / 3);
  LC_CHECK(nseq >= 0 && cu_seqlens[0] == 0 && cu_seqlens[nseq] == T, "attentionVarlen: cu_seqlens must run from 0 to T");
  for (int s = 0; s < nseq; s++) LC_CHECK(cu_seqlens[s + 1] >= cu_seqlens[s], "attentionVarlen: cu_seqlens must be non-decreasing");
  LcTensor* y = alloc(qkv->dtype, {T, (int64_t)H});
  std::vector<int4> tiles = kernel == 0 ? attention_tiles_tc(cu_seqlens, nseq) : attention_tiles(cu_seqlens, nseq);
  if (!tiles.empty()) {
    int4* d = (int4*)dmalloc(tiles.size() * sizeof(int4));
    CUDA_OK(cudaMemcpyAsync(d, tiles.data(), tiles.size() * sizeof(int4), cudaMemcpyHostToDevice, stream()));
    if (kernel == 0)
      attention_varlen_tc(qkv->data(), y->data(), d, (int)tiles.size(), T, H, half_window, (float)scale, qkv->dtype, stream());
    else
      attention_varlen(qkv->data(), y->data(), d, (int)tiles.size(), T, H, half_window, (float)scale, qkv->dtype, stream());
    dfree(d);
  }
  *out = handle(y);
  LC_API_END
}
