// Tensor-core GEMM for sm_100a: y[M, N] = x[M, K] · w[N, K]ᵀ with a fused epilogue.
//
// Replaces the reference's linear kernels (WGSL gemm*Kernel,
// packages/backend-webgpu/src/kernels.ts:648-918; MLX addmm/matmul,
// packages/backend-mlx/src/index.ts:576-587) for the contract op `linear`
// (packages/tensor-backend/src/index.ts:211-215: f32 accumulation).
//
// Design (one persistent CTA per SM, 10 warps):
//   warp 0      TMA producer: 128x64 tiles of x and BNx64 tiles of w, 128-byte
//               swizzle, into a STAGES-deep shared-memory ring (mbarrier full/empty);
//   warp 1      allocates TMEM and issues tcgen05.mma (M=128, N=BN, K=16,
//               fp16/bf16 in, f32 accumulate) from one elected thread; commits
//               free the ring slot and, per tile, signal the epilogue;
//   warps 2-9   epilogue: tcgen05.ld of the f32 accumulator (a warp reaches
//               the 32 TMEM lanes = rows of quarter warp % 4; warps w and
//               w + 4 share those rows and take one half of the tile's
//               columns each), fused bias / residual / RoPE / GeGLU /
//               folded-LayerNorm correction (and the row statistics a later
//               folded LayerNorm needs), 16-byte or TMA stores.
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue
// of tile i overlaps the main loop of tile i+1. Every mbarrier wait is bounded
// (2 s of %globaltimer); on timeout the kernel records an error word, drains
// its own in-flight copies and MMAs, frees TMEM and returns.
// No cluster launch and no multicast: each CTA loads its own tiles.
#include "lc_api.h"
#include "lc_gemm.h"
#include "lc_sm100.cuh"
#include "lc_quant.cuh"
#include "lc_gelu.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <map>
#include <tuple>

__device__ unsigned int g_gemm_err;

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
using namespace sm100;

struct GemmArgs {
  int M, N, K;
  int ntile_n, ntiles;
  void* y;
  int64_t ldy;
  int vec_ok;  // 16-byte stores allowed (ldy % 8 == 0)
  const void* bias;
  int bias_dtype;
  GemmEpilogue ep;
  int ksplit;  // split-K factor: the CTAs of a cluster of ksplit share a tile (k_gemm_tc with KS)
  GemmQuantB q;  // QB: the packed weight (tmB maps its bytes)
};

__device__ __forceinline__ float gelu_exact(float x) { return 0.5f * x * (1.0f + erff(x * 0.7071067811865476f)); }

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float2 v) {
  if constexpr (std::is_same<T, __half>::value) {
    __half2 h = __floats2half2_rn(v.x, v.y);
    return *(uint32_t*)&h;
  } else {
    __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
    return *(uint32_t*)&h;
  }
}

// Folded LayerNorm, consumer side: mean and 1/sqrt(var + eps) of row `row`
// from its per-part (mean, M2) statistics (Chan et al.'s pairwise combination).
// One pass over the parts, shifted by the first part's mean K for accuracy:
// S1 = Σ c_p·(mean_p − K), S2 = Σ (M2_p + c_p·(mean_p − K)²),
// mean = K + S1/n, M2 = S2 − S1²/n.
constexpr int LN_MAX_PARTS = 64;
__device__ __forceinline__ void ln_row(const GemmEpilogue& ep, int row, int M, float& mu, float& r) {
  mu = 0.f;
  r = 1.f;
  if (row >= M) return;
  const float2* st = ep.ln_stats + (int64_t)row * ep.ln_parts;
  const float inv_n = 1.f / (float)ep.ln_cols;
  const float k0 = st[0].x;
  float s1 = 0.f, s2 = 0.f;
  auto part = [&](int p, float2 v) {
    const float c = (float)min(ep.ln_part_cols, ep.ln_cols - p * ep.ln_part_cols), d = v.x - k0;
    s1 = fmaf(c, d, s1);
    s2 += fmaf(c * d, d, v.y);
  };
  if ((ep.ln_parts & 1) == 0) {  // two parts per 16-byte load (rows start 16-byte aligned)
    const float4* st4 = (const float4*)st;
#pragma unroll 8
    for (int p = 0; p < ep.ln_parts / 2; p++) {
      const float4 v = st4[p];
      part(2 * p, make_float2(v.x, v.y));
      part(2 * p + 1, make_float2(v.z, v.w));
    }
  } else {
#pragma unroll 8
    for (int p = 0; p < ep.ln_parts; p++) part(p, st[p]);
  }
  mu = fmaf(s1, inv_n, k0);
  r = rsqrtf(fmaxf(fmaf(-s1 * s1, inv_n, s2), 0.f) * inv_n + ep.ln_eps);
}
// acc columns [col, col+64) -> r·(acc − μ·wsum)
__device__ __forceinline__ void ln_apply(const GemmEpilogue& ep, int col, float mu, float r, float* a, float* b) {
  const float4* w4 = (const float4*)(ep.ln_wsum + col);
#pragma unroll
  for (int q = 0; q < 8; q++) {
    const float4 w = __ldg(w4 + q);
    a[q * 4 + 0] = r * fmaf(-mu, w.x, a[q * 4 + 0]);
    a[q * 4 + 1] = r * fmaf(-mu, w.y, a[q * 4 + 1]);
    a[q * 4 + 2] = r * fmaf(-mu, w.z, a[q * 4 + 2]);
    a[q * 4 + 3] = r * fmaf(-mu, w.w, a[q * 4 + 3]);
  }
#pragma unroll
  for (int q = 0; q < 8; q++) {
    const float4 w = __ldg(w4 + 8 + q);
    b[q * 4 + 0] = r * fmaf(-mu, w.x, b[q * 4 + 0]);
    b[q * 4 + 1] = r * fmaf(-mu, w.y, b[q * 4 + 1]);
    b[q * 4 + 2] = r * fmaf(-mu, w.z, b[q * 4 + 2]);
    b[q * 4 + 3] = r * fmaf(-mu, w.w, b[q * 4 + 3]);
  }
}
// a pair rounded to the stored 16-bit type and back (one packed conversion)
template <typename T>
__device__ __forceinline__ float2 round_pair(float x, float y) {
  if constexpr (std::is_same<T, __half>::value) return __half22float2(__floats2half2_rn(x, y));
  else return __bfloat1622float2(__floats2bfloat162_rn(x, y));
}
// two packed 16-bit values as floats
template <typename T>
__device__ __forceinline__ float2 unpack_pair(uint32_t u) {
  if constexpr (std::is_same<T, __half>::value) return __half22float2(*(const __half2*)&u);
  else return __bfloat1622float2(*(const __nv_bfloat162*)&u);
}
// Producer side: round the 64 outputs of a unit to the stored type (so the
// statistics describe the tensor the next layer reads) and return their
// (mean, M2), summed in four independent chains.
template <typename T>
__device__ __forceinline__ float2 stats_unit(float* a, float* b) {
  float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    const float2 ra = round_pair<T>(a[j], a[j + 1]), rb = round_pair<T>(b[j], b[j + 1]);
    a[j] = ra.x;
    a[j + 1] = ra.y;
    b[j] = rb.x;
    b[j + 1] = rb.y;
    s[0] += ra.x;
    s[1] += ra.y;
    s[2] += rb.x;
    s[3] += rb.y;
  }
  const float mu = ((s[0] + s[1]) + (s[2] + s[3])) * (1.f / 64.f);
  float q[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    const float d0 = a[j] - mu, d1 = a[j + 1] - mu, d2 = b[j] - mu, d3 = b[j + 1] - mu;
    q[0] = fmaf(d0, d0, q[0]);
    q[1] = fmaf(d1, d1, q[1]);
    q[2] = fmaf(d2, d2, q[2]);
    q[3] = fmaf(d3, d3, q[3]);
  }
  return make_float2(mu, (q[0] + q[1]) + (q[2] + q[3]));
}

// stats_unit on packed pairs (a[j] = columns col+2j, col+2j+1; b the same
// 32 columns on): the chains and their order are stats_unit's, so are the
// bits; half the instructions.
template <typename T>
__device__ __forceinline__ float2 stats_unit2(float2* a, float2* b) {
  float2 sa = make_float2(0.f, 0.f), sb = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 16; j++) {
    a[j] = round_pair<T>(a[j].x, a[j].y);
    b[j] = round_pair<T>(b[j].x, b[j].y);
    sa = add2(sa, a[j]);
    sb = add2(sb, b[j]);
  }
  const float mu = ((sa.x + sa.y) + (sb.x + sb.y)) * (1.f / 64.f);
  const float2 nmu = make_float2(-mu, -mu);
  float2 qa = make_float2(0.f, 0.f), qb = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 16; j++) {
    const float2 da = add2(a[j], nmu), db = add2(b[j], nmu);
    qa = fma2(da, da, qa);
    qb = fma2(db, db, qb);
  }
  return make_float2(mu, (qa.x + qa.y) + (qb.x + qb.y));
}

// store 32 consecutive values v[0..31] at columns [col, col+32) of row `row`, valid columns < ncols
template <typename T>
__device__ __forceinline__ void store32(T* rowp, int col, int ncols, const float* v, bool vec) {
  if (vec && col + 32 <= ncols) {
#pragma unroll
    for (int q = 0; q < 4; q++) {
      uint4 u;
      T* h = (T*)&u;
#pragma unroll
      for (int j = 0; j < 8; j++) h[j] = TcFmt<T>::cvt(v[q * 8 + j]);
      *(uint4*)(rowp + col + q * 8) = u;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; j++)
      if (col + j < ncols) rowp[col + j] = TcFmt<T>::cvt(v[j]);
  }
}

template <typename T>
__device__ __forceinline__ void load32f(const T* p, int col, int ncols, float* v, bool vec) {
  if (vec && col + 32 <= ncols) {
#pragma unroll
    for (int q = 0; q < 4; q++) {
      uint4 u = *(const uint4*)(p + col + q * 8);
      const T* h = (const T*)&u;
#pragma unroll
      for (int j = 0; j < 8; j++) v[q * 8 + j] = TcFmt<T>::back(h[j]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = (col + j < ncols) ? TcFmt<T>::back(p[col + j]) : 0.f;
  }
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"((uint64_t)map), "r"(smem_u32(src)),
               "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Epilogue warps (two per TMEM lane quarter) and their staging: one 4 KB
// buffer per warp holding a 32-row x 64-column block in the 128-byte-swizzled
// layout the TMA store/load tensor maps use (16-byte chunk c of row r at
// chunk position c ^ (r & 7)).
constexpr int EPI_WARPS = 8;                    // single-CTA kernel
constexpr int GEMM_THREADS = 64 + 32 * EPI_WARPS;
constexpr uint32_t STG_BYTES = EPI_WARPS * 4096;
constexpr int PAIR_EPI_WARPS = 8;               // CTA-pair kernel: two staging buffers per warp
constexpr int PAIR_NBUF = 2;
constexpr int PAIR_THREADS = 64 + 32 * PAIR_EPI_WARPS;

// split-K partial tile: BM rows of BN f32 accumulators, rows padded by 16 bytes
template <int BN>
constexpr uint32_t part_bytes() {
  return BM * (BN + 4) * 4;
}
// QB: packed weight block of one stage (BN rows of BK values, at most 8 bits each)
template <int BN>
constexpr uint32_t packed_bytes() {
  return BN * BK;
}
template <int STAGES, int BN>
constexpr size_t gemm_smem_bytes(bool tma_epi, bool ksplit = false, bool qb = false) {
  return (size_t)STAGES * (BM * BK * 2 + BN * BK * 2 + (qb ? packed_bytes<BN>() : 0)) + (tma_epi ? STG_BYTES : 0) +
         (ksplit ? part_bytes<BN>() : 0) + 1024 + 512;
}

// QB: the epilogue warps turn a stage's packed weight block (BN rows x BK
// values; rows >= N and columns >= K arrive as zero bytes) into the MMA's
// 16-bit operand in the 128-byte-swizzled K-major layout a TMA load would
// produce: 16-byte chunk c (values 8c..8c+7) of row r at r·128 + ((c ^ (r&7))·16).
// Thread et takes chunks (r, c) = divmod(et + 32·EPI_WARPS·i, 8).
// Each value equals what the dense dequantisation kernels store
// (dequant_rounded, then the optional column scale in f32 and one rounding),
// so the product is bit-identical to dequantising first. For f16 scales,
// biases and output the value is one fma.rn.f16x2: q (|q| <= 255), s and b
// are exact in f16, so q·s + b is an exact multiple of 2^-24 below 2^24 — at
// most 48 significant bits, exact in the f64 form too — and both round it
// once to f16.
template <int BN>
constexpr int conv_tasks() {
  return BN * 8 / (32 * EPI_WARPS);
}
// the scale and bias of each of this thread's chunks of K block kb (issued before the block lands)
template <int BN>
__device__ __forceinline__ void load_packed_scales(const GemmArgs& args, int n0, int kb, int et, float2* sb) {
  const GemmQuantB& q = args.q;
  const int64_t G = (args.K + q.group - 1) / q.group;
  const int nrows = args.N * (args.ep.kind == EPI_GEGLU ? 2 : 1);
#pragma unroll
  for (int i = 0; i < conv_tasks<BN>(); i++) {
    const int task = et + 32 * EPI_WARPS * i, r = task >> 3, c = task & 7;
    const int n = n0 + r, k = kb * BK + 8 * c;
    sb[i] = make_float2(0.f, 0.f);
    if (n < nrows && k < args.K) {
      const int64_t gi = (int64_t)n * G + k / q.group;
      sb[i].x = ld_as<float>((const char*)q.scales, q.sdt, gi);
      sb[i].y = q.biases ? ld_as<float>((const char*)q.biases, q.sdt, gi) : 0.f;
    }
  }
}
template <typename T, int BN>
__device__ __forceinline__ void convert_packed_block(const GemmArgs& args, const uint8_t* pk, uint8_t* sb_out, int n0, int kb, int et,
                                                     const float2* sb) {
  const GemmQuantB& q = args.q;
  const int bits = q.bits, rowb = BK * bits / 8;
  const int nrows = args.N * (args.ep.kind == EPI_GEGLU ? 2 : 1);
  constexpr bool HALF = std::is_same<T, __half>::value;
  const bool fast = HALF && q.sdt == LC_F16;
#pragma unroll
  for (int i = 0; i < conv_tasks<BN>(); i++) {
    const int task = et + 32 * EPI_WARPS * i, r = task >> 3, c = task & 7;
    const int n = n0 + r, k = kb * BK + 8 * c;
    uint4 out = make_uint4(0u, 0u, 0u, 0u);
    if (n < nrows && k < args.K) {
      const uint8_t* src = pk + r * rowb + c * bits;  // 8 values: 4 or 8 bytes
      const uint64_t raw = bits == 4 ? (uint64_t)*(const uint32_t*)src : *(const uint64_t*)src;
      int qv[8];
#pragma unroll
      for (int j = 0; j < 8; j++) {
        if (bits == 4) {
          const int nib = (int)((raw >> (4 * j)) & 15u);
          qv[j] = q.mode == 0 ? ((nib ^ 8) - 8) : nib;
        } else {
          const int byte = (int)((raw >> (8 * j)) & 255u);
          qv[j] = q.mode == 0 ? (int)(int8_t)byte : byte;
        }
      }
      const bool full8 = k + 8 <= args.K;
      if (fast && full8) {
        const __half2 s2 = __float2half2_rn(sb[i].x), b2 = __float2half2_rn(sb[i].y);  // exact: f16 values
        __half2 h[4];
#pragma unroll
        for (int j = 0; j < 4; j++) h[j] = __hfma2(__halves2half2(__int2half_rn(qv[2 * j]), __int2half_rn(qv[2 * j + 1])), s2, b2);
        if (q.gamma) {
          const float4 g0 = __ldg((const float4*)(q.gamma + k)), g1 = __ldg((const float4*)(q.gamma + k + 4));
          const float2 gg[4] = {make_float2(g0.x, g0.y), make_float2(g0.z, g0.w), make_float2(g1.x, g1.y), make_float2(g1.z, g1.w)};
#pragma unroll
          for (int j = 0; j < 4; j++) h[j] = __float22half2_rn(mul2(__half22float2(h[j]), gg[j]));
        }
        out = *(const uint4*)h;
      } else {
        const int odt = HALF ? LC_F16 : LC_BF16;
        T v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
          float d = 0.f;
          if (k + j < args.K) {
            d = dequant_rounded(odt, qv[j], sb[i].x, sb[i].y);
            if (q.gamma) d = d * __ldg(q.gamma + k + j);
          }
          v[j] = TcFmt<T>::cvt(d);
        }
        out = *(const uint4*)v;
      }
    }
    *(uint4*)(sb_out + r * 128 + ((c ^ (r & 7)) << 4)) = out;
  }
}

// The TMA-store epilogue of both GEMM kernels (warps 2..9 of the CTA). Tiles
// t = t_begin, t_begin + t_step, ...; this CTA's rows of tile t start at
// (t / ntile_n) * tile_rows + row_off. In a CTA pair the accumulator-free
// arrivals go to the barrier of CTA 0, whose thread issues the MMAs.
//
// EW epilogue warps (2 .. EW+1), EW/4 per TMEM lane quarter warp % 4. Each
// warp owns 32 rows and a contiguous share of the tile's 64-column units (a
// GeGLU output block, an even/odd unit pair, stays in one warp). Per unit:
// tcgen05.ld the f32 accumulators, apply folded LayerNorm / RoPE / bias /
// residual / GeGLU (packed f32 pairs), write the row's 8 chunks into a
// swizzled staging buffer, and one lane issues a TMA store of the 32 x 64
// block (rows >= M and columns >= N are clipped by the tensor map). The
// residual block arrives by TMA load into the buffer its result is stored
// from; when the warp has a buffer per unit (NBUF staging buffers) all its
// residual blocks are requested before the tile's accumulator is ready, and
// with two buffers a store drains while the next unit computes. The tile's
// LayerNorm statistics and the first unit's LayerNorm column sums (one
// coalesced load per warp, shared by shuffles) are read ahead as well.
//
// Split K (KS, args.ksplit = S > 1, one tile per cluster): the S CTAs of a
// cluster computed partial accumulators of the same tile over S slices of K.
// CTA r owns the lane quarters q with q·S/4 == r. For each quarter, the warp
// holding whole rows of the tile copies its partial rows from TMEM into this
// CTA's shared memory (sSend, the idle pipeline stages) and one bulk copy
// moves them into the owner's receive buffer (sP: one slot of 128/S rows per
// CTA of the cluster), completing on the owner's pbar[0], which expects
// 128 rows' worth of bytes. The owner's warps then add the S slots of their
// rows in the fixed order 0..S-1 (the same bits whichever CTA is slower), put
// the sums back into TMEM and run the ordinary epilogue on the sums.
template <typename T, int BN, bool PAIR, int EW, int NBUF, bool KS = false>
__device__ __forceinline__ void epilogue_tma(const GemmArgs& args, const CUtensorMap* tmYp, const CUtensorMap* tmRp, uint8_t* sE, uint64_t* rbar,
                                             uint64_t* tfull, uint64_t* tempty, volatile int* abort, uint32_t tmem, int warp, int lane,
                                             int t_begin, int t_step, int tile_rows, int row_off, float* sP = nullptr,
                                             float* sSend = nullptr, uint64_t* pbar = nullptr) {
  const CUtensorMap& tmY = *tmYp;
  const CUtensorMap& tmR = *tmRp;
  constexpr int NSUB = EW / 4;  // warps per lane quarter
  const int quarter = warp & 3, sub = (warp - 2) >> 2;
  const GemmEpilogue& ep = args.ep;
  const bool geglu = ep.kind == EPI_GEGLU;
  const bool resid = ep.kind == EPI_RESIDUAL;
  const int ncols = geglu ? 2 * args.N : args.N;  // accumulator columns that hold data
  constexpr int U = BN / 64;
  int u_lo, u_hi;
  if (geglu) {
    const int per = (U / 2) / NSUB > 0 ? (U / 2) / NSUB : 1, b0 = sub * per;
    u_lo = min(U, 2 * b0);
    u_hi = min(U, 2 * (b0 + per));
  } else {
    const int per = U / NSUB > 0 ? U / NSUB : 1;
    u_lo = min(U, sub * per);
    u_hi = min(U, u_lo + per);
  }
  // residual blocks requested ahead: one buffer per unit of this warp
  const bool ahead = resid && u_hi - u_lo <= NBUF;
  const int nparts = args.N / 64;  // row statistics: one (mean, M2) per 64-column unit
  uint8_t* stg0 = sE + (warp - 2) * NBUF * 4096;
  uint64_t* rb0 = rbar + (warp - 2) * NBUF;
  uint32_t rph[NBUF];
#pragma unroll
  for (int i = 0; i < NBUF; i++) rph[i] = 0;
  int acc = 0;
  uint32_t acc_phase = 0;
  bool ok = true;
  uint32_t nstore = 0;  // TMA stores issued by this warp
  const uint32_t tempty0 = PAIR ? mapa_rank(smem_u32(tempty), 0) : 0;  // CTA 0's accumulator-empty barriers
  const int S = KS ? args.ksplit : 1;
  const bool split = KS && S > 1;
  const bool mine = !split || (quarter * S) / 4 == (int)cluster_rank();  // this warp's rows are reduced here
  for (int t = t_begin; t < args.ntiles && ok; t += t_step) {
    const int m0 = (t / args.ntile_n) * tile_rows + row_off, n0 = (t % args.ntile_n) * BN;
    const int row0 = m0 + quarter * 32;
    const int row = row0 + lane;
    const bool live = row < args.M;
    float ln_mu = 0.f, ln_r = 1.f;
    if (ep.ln_stats && mine) ln_row(ep, row, args.M, ln_mu, ln_r);
    const bool rope = ep.kind == EPI_ROPE_QKV && n0 + u_lo * 64 < ep.rope_cols;
    // this row's RoPE factors: table [16][cap] of (cos 2i, cos 2i+1, sin 2i, sin 2i+1)
    const float4* rq = (const float4*)ep.rope_cs + (rope && live ? ep.pos[row] : 0);
    // the first unit's LayerNorm column sums (lane l: columns 2l, 2l+1)
    float2 wsp = make_float2(0.f, 0.f);
    if (ep.ln_stats && mine && n0 + u_lo * 64 < ncols) wsp = __ldg((const float2*)(ep.ln_wsum + n0 + u_lo * 64) + lane);
    if (ahead && mine) {  // the residual blocks, in flight while the accumulator is computed
      if (lane == 0) bulk_wait_read0();  // earlier stores have read the buffers
      __syncwarp();
      if (lane == 0)
        for (int i = 0; i < NBUF && u_lo + i < u_hi && n0 + (u_lo + i) * 64 < ncols; i++) {
          mbar_arrive_expect_tx(&rb0[i], 4096);
          tma_load_2d(stg0 + i * 4096, &tmR, &rb0[i], n0 + (u_lo + i) * 64, row0);
        }
    }
    if (!mbar_wait(&tfull[acc], acc_phase, abort, &g_gemm_err)) break;
    tc_fence_after();
    const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
    if constexpr (KS) {
      if (split) {
        // rows of lane quarter q are reduced by CTA q·S/4, which holds one
        // slot of 128/S rows per CTA of the cluster
        const int owner = (quarter * S) / 4, orows = BM / S;
        const int lrow0 = (quarter - owner * (4 / S)) * 32;
        if (u_lo == 0 && u_hi == U) {  // this warp holds whole rows of the tile: it sends the quarter
          float* srow = sSend + (quarter * 32 + lane) * (BN + 4);
#pragma unroll 1
          for (int u = 0; u < U; u++) {
            uint32_t ra[32], rbv[32];
            tmem_ld32(tbase + u * 64, ra);
            tmem_ld32(tbase + u * 64 + 32, rbv);
            tmem_wait_ld();
            float4* p4 = (float4*)(srow + u * 64);
#pragma unroll
            for (int j = 0; j < 8; j++) {
              p4[j] = make_float4(__uint_as_float(ra[4 * j]), __uint_as_float(ra[4 * j + 1]), __uint_as_float(ra[4 * j + 2]),
                                  __uint_as_float(ra[4 * j + 3]));
              p4[8 + j] = make_float4(__uint_as_float(rbv[4 * j]), __uint_as_float(rbv[4 * j + 1]), __uint_as_float(rbv[4 * j + 2]),
                                      __uint_as_float(rbv[4 * j + 3]));
            }
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0)
            bulk_copy_to_cluster(mapa_rank(smem_u32(sP + ((int)cluster_rank() * orows + lrow0) * (BN + 4)), (uint32_t)owner),
                                 smem_u32(sSend + quarter * 32 * (BN + 4)), 32u * (BN + 4) * 4u,
                                 mapa_rank(smem_u32(&pbar[0]), (uint32_t)owner));
        }
        if (!mine) {  // another CTA reduces these rows
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[acc]);
          if (++acc == 2) { acc = 0; acc_phase ^= 1; }
          continue;
        }
        if (!mbar_wait(&pbar[0], 0, abort, &g_gemm_err)) break;
        // sum the S slots of this row in the order 0, 1, ..., S-1
        const float* p0 = sP + (lrow0 + lane) * (BN + 4);
#pragma unroll 1
        for (int u = u_lo; u < u_hi; u++) {
#pragma unroll
          for (int h = 0; h < 2; h++) {  // columns [32h, 32h+32) of the unit
            const float4* src = (const float4*)(p0 + u * 64 + 32 * h);
            float4 v[8];
#pragma unroll
            for (int j = 0; j < 8; j++) v[j] = src[j];
            for (int c = 1; c < S; c++) {
              const float4* sc = src + c * orows * (BN + 4) / 4;
#pragma unroll
              for (int j = 0; j < 8; j++) {
                const float4 w = sc[j];
                v[j].x += w.x;
                v[j].y += w.y;
                v[j].z += w.z;
                v[j].w += w.w;
              }
            }
            uint32_t r[32];
#pragma unroll
            for (int j = 0; j < 8; j++) {
              r[4 * j] = __float_as_uint(v[j].x);
              r[4 * j + 1] = __float_as_uint(v[j].y);
              r[4 * j + 2] = __float_as_uint(v[j].z);
              r[4 * j + 3] = __float_as_uint(v[j].w);
            }
            tmem_st32(tbase + u * 64 + 32 * h, r);
          }
        }
        tmem_wait_st();
      }
    }
    // The accumulator buffer is handed back to the MMA warp as soon as this
    // warp has read its last unit into registers (the rest of the epilogue
    // works from registers and shared memory).
    bool released = false;
    auto release = [&]() {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR && row_off != 0) mbar_arrive_cluster(tempty0 + 8 * acc);  // the pair's MMA runs in CTA 0
        else mbar_arrive(&tempty[acc]);
      }
      released = true;
    };
#pragma unroll 1
    for (int u = u_lo; u < u_hi; u++) {
      const int col = n0 + u * 64;
      const bool first = !geglu || (u & 1) == 0;  // GeGLU: two units fill one 64-column output block
      const bool last = !geglu || (u & 1) == 1;
      const int bcol = geglu ? n0 + (u & ~1) * 64 : col;  // first accumulator column of the block
      if (bcol >= ncols) break;  // the rest of this tile is past the weight rows
      const bool more = u + 1 < u_hi && (geglu ? n0 + ((u + 1) & ~1) * 64 : col + 64) < ncols;
      // staging buffer: the unit's residual buffer (loaded ahead), the one, or
      // alternating with this warp's stores
      const int bi = ahead ? u - u_lo : (NBUF == 1 ? 0 : (int)(nstore & 1));
      uint8_t* stg = stg0 + bi * 4096;
      if (!ahead && first && resid) {  // the residual block lands in the staging buffer
        if (lane == 0) bulk_wait_read0();  // this warp's previous store has read the buffer
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_expect_tx(&rb0[0], 4096);
          tma_load_2d(stg, &tmR, &rb0[0], col, row0);
        }
      }
      uint32_t racc[64];
      tmem_ld64(tbase + u * 64, racc);
      tmem_wait_ld();
      // the last unit this warp reads: the loop ends after it, or the next unit (output block) is past the weight rows
      const bool last_ld = u + 1 >= u_hi ||
                           (geglu ? ((u & 1) == 0 ? bcol + 64 >= ncols : n0 + ((u + 1) & ~1) * 64 >= ncols) : col + 64 >= ncols);
      if (last_ld) release();
      // a = accumulator columns col..col+31, b = col+32..col+63, as packed pairs
      float2 a[16], b[16];
#pragma unroll
      for (int j = 0; j < 16; j++) {
        a[j] = make_float2(__uint_as_float(racc[2 * j]), __uint_as_float(racc[2 * j + 1]));
        b[j] = make_float2(__uint_as_float(racc[32 + 2 * j]), __uint_as_float(racc[32 + 2 * j + 1]));
      }
      if (ep.ln_stats) {  // r·(acc − μ·wsum); wsum of columns col+2j, col+2j+1 sits in lane j
        const float2 nmu = make_float2(-ln_mu, -ln_mu), r2 = make_float2(ln_r, ln_r);
#pragma unroll
        for (int j = 0; j < 16; j++) {
          const float2 wa = make_float2(__shfl_sync(0xffffffffu, wsp.x, j), __shfl_sync(0xffffffffu, wsp.y, j));
          const float2 wb = make_float2(__shfl_sync(0xffffffffu, wsp.x, 16 + j), __shfl_sync(0xffffffffu, wsp.y, 16 + j));
          a[j] = mul2(r2, fma2(nmu, wa, a[j]));
          b[j] = mul2(r2, fma2(nmu, wb, b[j]));
        }
        if (more) wsp = __ldg((const float2*)(ep.ln_wsum + col + 64) + lane);
      }
      if (geglu) {
#pragma unroll
        for (int j = 0; j < 16; j++) a[j] = mul2(gelu_as2(a[j]), b[j]);
      } else {
        if (rope && col < ep.rope_cols) {  // (x1, x2) -> (x1·cos − x2·sin, x2·cos + x1·sin)
#pragma unroll
          for (int j = 0; j < 16; j++) {
            const float4 v = __ldg(rq + (int64_t)j * ep.rope_cap);
            const float2 c = make_float2(v.x, v.y), sn = make_float2(v.z, v.w), nsn = make_float2(-v.z, -v.w);
            const float2 x1 = a[j], x2 = b[j];
            a[j] = fma2(x2, nsn, mul2(x1, c));
            b[j] = fma2(x1, sn, mul2(x2, c));
          }
        }
        if (args.bias) {
#pragma unroll
          for (int j = 0; j < 16; j++) {
            const int c0 = col + 2 * j;
            if (c0 < args.N) a[j].x += ld_as<float>((const char*)args.bias, args.bias_dtype, c0);
            if (c0 + 1 < args.N) a[j].y += ld_as<float>((const char*)args.bias, args.bias_dtype, c0 + 1);
            if (c0 + 32 < args.N) b[j].x += ld_as<float>((const char*)args.bias, args.bias_dtype, c0 + 32);
            if (c0 + 33 < args.N) b[j].y += ld_as<float>((const char*)args.bias, args.bias_dtype, c0 + 33);
          }
        }
        if (resid) {
          if (!mbar_wait(&rb0[bi], rph[bi], abort, &g_gemm_err)) { ok = false; break; }
          rph[bi] ^= 1;
#pragma unroll
          for (int c = 0; c < 8; c++) {
            uint4 v = *(const uint4*)(stg + lane * 128 + ((c ^ (lane & 7)) << 4));
            const uint32_t* hw = (const uint32_t*)&v;
            float2* dst = c < 4 ? a + c * 4 : b + (c - 4) * 4;
#pragma unroll
            for (int j = 0; j < 4; j++) dst[j] = add2(dst[j], unpack_pair<T>(hw[j]));
          }
          if (ep.stats_out && live) ep.stats_out[(int64_t)row * nparts + col / 64] = stats_unit2<T>(a, b);
        }
      }
      if (first && !resid) {  // the store that last used this buffer has read it
        if (lane == 0) {
          if (NBUF == 1) bulk_wait_read0();
          else bulk_wait_read1();
        }
        __syncwarp();
      }
      // write this row's chunks: GeGLU writes 4 chunks (32 columns) per unit, else 8
      const int c0 = geglu ? (u & 1) * 4 : 0;
#pragma unroll
      for (int c = 0; c < 8; c++) {
        if (geglu && c >= 4) break;
        const float2* src = (c < 4) ? a + c * 4 : b + (c - 4) * 4;
        uint4 v;
        uint32_t* h = (uint32_t*)&v;
#pragma unroll
        for (int j = 0; j < 4; j++) h[j] = pack_pair<T>(src[j]);
        const int cc = c0 + c;
        *(uint4*)(stg + lane * 128 + ((cc ^ (lane & 7)) << 4)) = v;
      }
      if (last || bcol + 64 >= ncols) {
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmY, stg, geglu ? bcol / 2 : col, row0);
          bulk_commit();
        }
        nstore++;
        if (geglu && (u & 1) == 0) break;  // the pair's second unit is past the weight rows
      }
    }
    if (!released) release();
    if (++acc == 2) { acc = 0; acc_phase ^= 1; }
  }
  if (lane == 0) bulk_wait_all();
  __syncwarp();
}

// Split K (KS with args.ksplit = S > 1; one tile per cluster). The partial
// tiles meet in the owners' shared memory as in epilogue_tma — the warp
// holding a lane quarter's rows sends them with one bulk copy to the CTA that
// reduces that quarter — but the owner's rows (128/S of them) are then
// finished by all EW epilogue warps together instead of one warp per lane
// quarter: a warp takes R rows at a time (R = 4 for 64-column tiles, 2 for
// GeGLU's 128), lane = (row, 8-column chunk), sums the S slots of its chunk
// in the order 0..S-1, applies the epilogue to its 8 values (the RoPE / GeGLU
// partner half of the 64-column unit is four lanes away), stages the R rows
// and stores them with one TMA store (the y map's box is 64 columns x R rows).
// The row statistics of a residual epilogue reduce over the unit's 8 lanes.
template <typename T, int BN, int EW>
__device__ __forceinline__ void epilogue_split(const GemmArgs& args, const CUtensorMap* tmYp, uint8_t* sE, uint64_t* tfull,
                                               uint64_t* tempty, volatile int* abort, uint32_t tmem, int warp, int lane, float* sP,
                                               float* sSend, uint64_t* pbar) {
  const GemmEpilogue& ep = args.ep;
  const int S = args.ksplit, rank = (int)cluster_rank(), orows = BM / S;
  const int quarter = warp & 3, sub = (warp - 2) >> 2;
  constexpr int U = BN / 64;
  const bool geglu = ep.kind == EPI_GEGLU, resid = ep.kind == EPI_RESIDUAL;
  const int t = blockIdx.x / S;  // the cluster's tile
  const int m0 = (t / args.ntile_n) * BM, n0 = (t % args.ntile_n) * BN;
  bool ok = mbar_wait(&tfull[0], 0, abort, &g_gemm_err);
  if (ok) {
    tc_fence_after();
    if (sub == 0) {  // this quarter's 32 rows of the partial tile -> the owner's slot for this CTA
      const int owner = (quarter * S) / 4, lrow0 = (quarter - owner * (4 / S)) * 32;
      const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16);
      float* srow = sSend + (quarter * 32 + lane) * (BN + 4);
#pragma unroll 1
      for (int u = 0; u < U; u++) {
        uint32_t ra[32], rb[32];
        tmem_ld32(tbase + u * 64, ra);
        tmem_ld32(tbase + u * 64 + 32, rb);
        tmem_wait_ld();
        float4* p4 = (float4*)(srow + u * 64);
#pragma unroll
        for (int j = 0; j < 8; j++) {
          p4[j] = make_float4(__uint_as_float(ra[4 * j]), __uint_as_float(ra[4 * j + 1]), __uint_as_float(ra[4 * j + 2]),
                              __uint_as_float(ra[4 * j + 3]));
          p4[8 + j] = make_float4(__uint_as_float(rb[4 * j]), __uint_as_float(rb[4 * j + 1]), __uint_as_float(rb[4 * j + 2]),
                                  __uint_as_float(rb[4 * j + 3]));
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0)
        bulk_copy_to_cluster(mapa_rank(smem_u32(sP + (rank * orows + lrow0) * (BN + 4)), (uint32_t)owner),
                             smem_u32(sSend + quarter * 32 * (BN + 4)), 32u * (BN + 4) * 4u, mapa_rank(smem_u32(&pbar[0]), (uint32_t)owner));
    }
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(&tempty[0]);  // the accumulator has been read (one tile per CTA)
  constexpr int CPR = BN / 8;    // 8-column chunks per row of the tile
  constexpr int R = 32 / CPR;    // rows per warp pass
  const int k = lane % CPR, rl = lane / CPR;
  const int col = k * 8, unit = col / 64, uc = col % 64;  // tile column, its 64-column unit and place in it
  const int gc = n0 + col;                                // accumulator column
  const bool rope = ep.kind == EPI_ROPE_QKV && n0 + unit * 64 < ep.rope_cols;
  const int nparts = args.N / 64;
  float wsum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (ep.ln_stats && gc < (geglu ? 2 * args.N : args.N)) {  // a GeGLU tile may run past the weight rows
    const float4 w0 = __ldg((const float4*)(ep.ln_wsum + gc)), w1 = __ldg((const float4*)(ep.ln_wsum + gc) + 1);
    wsum[0] = w0.x, wsum[1] = w0.y, wsum[2] = w0.z, wsum[3] = w0.w, wsum[4] = w1.x, wsum[5] = w1.y, wsum[6] = w1.z, wsum[7] = w1.w;
  }
  float bias[8];
#pragma unroll
  for (int i = 0; i < 8; i++)
    bias[i] = (args.bias && !geglu && gc + i < args.N) ? ld_as<float>((const char*)args.bias, args.bias_dtype, gc + i) : 0.f;
  uint8_t* stg0 = sE + (warp - 2) * 4096;  // this warp's 4 KB of staging: two 1024-aligned buffers of R rows
  int npass = 0;
  bool waited = false;
#pragma unroll 1
  for (int r0 = (warp - 2) * R; r0 < orows; r0 += EW * R, npass++) {
    const int lr = r0 + rl, row = m0 + rank * orows + lr;
    const bool live = row < args.M;
    float mu = 0.f, rr = 1.f;
    if (ep.ln_stats) ln_row(ep, row, args.M, mu, rr);
    float res[8];
    if (resid) {
      uint4 rv = make_uint4(0u, 0u, 0u, 0u);
      if (live && gc < args.N) rv = __ldg((const uint4*)((const T*)ep.resid + (int64_t)row * ep.ldr + gc));
      const uint32_t* hw = (const uint32_t*)&rv;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float2 f = unpack_pair<T>(hw[j]);
        res[2 * j] = f.x;
        res[2 * j + 1] = f.y;
      }
    }
    float4 cs[4];
    if (rope) {
      const float4* rq = (const float4*)ep.rope_cs + (live ? ep.pos[row] : 0);
#pragma unroll
      for (int j = 0; j < 4; j++) cs[j] = __ldg(rq + (int64_t)(((uc % 32) >> 1) + j) * ep.rope_cap);
    }
    if (!waited) {
      ok = ok && mbar_wait(&pbar[0], 0, abort, &g_gemm_err);
      waited = true;
    }
    // the S slots of this chunk, added in the order 0..S-1
    float v[8];
    {
      const float4* src = (const float4*)(sP + lr * (BN + 4) + col);
      float4 x0 = src[0], x1 = src[1];
      for (int c = 1; c < S; c++) {
        const float4* sc = src + c * orows * (BN + 4) / 4;
        const float4 y0 = sc[0], y1 = sc[1];
        x0.x += y0.x, x0.y += y0.y, x0.z += y0.z, x0.w += y0.w;
        x1.x += y1.x, x1.y += y1.y, x1.z += y1.z, x1.w += y1.w;
      }
      v[0] = x0.x, v[1] = x0.y, v[2] = x0.z, v[3] = x0.w, v[4] = x1.x, v[5] = x1.y, v[6] = x1.z, v[7] = x1.w;
    }
    if (ep.ln_stats)
#pragma unroll
      for (int i = 0; i < 8; i++) v[i] = rr * fmaf(-mu, wsum[i], v[i]);
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; i++) o[i] = __shfl_xor_sync(0xffffffffu, v[i], 4);  // the other half of the unit
    const bool lo_half = uc < 32;
    uint4 packed;
    uint32_t* pk = (uint32_t*)&packed;
    if (geglu) {  // lanes of the gate half: gelu(gate) * up
#pragma unroll
      for (int j = 0; j < 4; j++) pk[j] = pack_pair<T>(mul2(gelu_as2(make_float2(v[2 * j], v[2 * j + 1])), make_float2(o[2 * j], o[2 * j + 1])));
    } else {
      if (rope) {  // (x1, x2) -> (x1 cos - x2 sin, x2 cos + x1 sin)
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float4 q = cs[j];
          if (lo_half) {
            v[2 * j] = fmaf(o[2 * j], -q.z, v[2 * j] * q.x);
            v[2 * j + 1] = fmaf(o[2 * j + 1], -q.w, v[2 * j + 1] * q.y);
          } else {
            v[2 * j] = fmaf(o[2 * j], q.z, v[2 * j] * q.x);
            v[2 * j + 1] = fmaf(o[2 * j + 1], q.w, v[2 * j + 1] * q.y);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 8; i++) v[i] += bias[i];
      if (resid)
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] += res[i];
#pragma unroll
      for (int j = 0; j < 4; j++) pk[j] = pack_pair<T>(make_float2(v[2 * j], v[2 * j + 1]));
      if (resid && ep.stats_out) {  // (mean, M2) of the stored unit: this lane's 8 values, then the unit's 8 lanes
        float f[8], sum = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float2 g = unpack_pair<T>(pk[j]);
          f[2 * j] = g.x;
          f[2 * j + 1] = g.y;
          sum += g.x + g.y;
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        const float m = sum * (1.f / 64.f);
        float q2 = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) q2 = fmaf(f[i] - m, f[i] - m, q2);
        q2 += __shfl_xor_sync(0xffffffffu, q2, 1);
        q2 += __shfl_xor_sync(0xffffffffu, q2, 2);
        q2 += __shfl_xor_sync(0xffffffffu, q2, 4);
        if (uc == 0 && live) ep.stats_out[(int64_t)row * nparts + gc / 64] = make_float2(m, q2);
      }
    }
    // stage the R rows (128-byte swizzle) and store them
    uint8_t* stg = stg0 + (npass & 1) * 2048;
    if (lane == 0) bulk_wait_read1();  // the store that last read this buffer is done with it
    __syncwarp();
    if (!geglu) *(uint4*)(stg + rl * 128 + ((k ^ (rl & 7)) << 4)) = packed;
    else if (lo_half) {
      const int oc = unit * 4 + uc / 8;  // output chunk: units 0 / 1 fill columns [0, 32) / [32, 64)
      *(uint4*)(stg + rl * 128 + ((oc ^ (rl & 7)) << 4)) = packed;
    }
    fence_async_smem();
    __syncwarp();
    const int srow = m0 + rank * orows + r0;
    if (lane == 0 && ok && srow < args.M) {
      tma_store_2d(tmYp, stg, geglu ? n0 / 2 : n0, srow);
      bulk_commit();
    }
  }
  if (!waited) mbar_wait(&pbar[0], 0, abort, &g_gemm_err);  // every partial sent here has landed before the CTA exits
  if (lane == 0) bulk_wait_all();
  __syncwarp();
}

// KS: split K over the CTAs of a cluster of args.ksplit (launched with that
// cluster size, one K slice per CTA rank): the unit of work is (tile, slice),
// CTA rank r takes K blocks [r·KB/S, (r+1)·KB/S) of its cluster's tiles and
// the epilogue reduces the partial tiles through distributed shared memory.
//
// QB: the weight is packed 4/8-bit (args.q; tmB maps its bytes). The producer
// loads the packed blocks (pfull) beside the activation blocks (full); the
// epilogue warps, idle until the accumulator is ready, dequantise each block
// into the stage's 16-bit operand (convert_packed_block) and arrive on
// conv[stage], which the MMA issuer waits for as well. The packed weight is
// resident, so its first blocks are requested and converted before the
// dependency wait. One unit of work per CTA.
template <typename T, int BN, int STAGES, bool TMAE, bool KS = false, bool QB = false>
__global__ void __launch_bounds__(GEMM_THREADS, 1) k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                                                    const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmR,
                                                    const __grid_constant__ GemmArgs args) {
  static_assert(!KS || TMAE, "split K runs with the TMA-store epilogue");
  extern __shared__ uint8_t smem_raw[];
  constexpr uint32_t A_BYTES = BM * BK * 2;
  constexpr uint32_t B_BYTES = BN * BK * 2;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  constexpr uint32_t PK_BYTES = QB ? packed_bytes<BN>() : 0;  // packed stage buffer (QB)
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sPk = sB + STAGES * B_BYTES;
  uint8_t* sE = sPk + STAGES * PK_BYTES;  // epilogue staging (TMAE only), 1024-aligned
  float* sP = (float*)(sE + (TMAE ? STG_BYTES : 0));  // split-K partial tile (KS only)
  uint64_t* full = (uint64_t*)((uint8_t*)sP + (KS ? part_bytes<BN>() : 0));
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* rbar = tempty + 2;  // residual-load barriers, one per epilogue warp
  uint64_t* pbar = rbar + EPI_WARPS;  // KS: the partial slots of this CTA's rows have landed
  uint64_t* pfull = pbar + 1;                  // QB: packed block landed
  uint64_t* conv = pfull + (QB ? STAGES : 0);  // QB: 16-bit operand written
  uint32_t* tmem_slot = (uint32_t*)(conv + (QB ? STAGES : 0));
  volatile int* abort = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = (args.K + BK - 1) / BK;
  const int S = KS ? args.ksplit : 1;
  static_assert(!QB || (KS && TMAE), "the packed-weight GEMM runs as the split-K instance");
  static_assert(PK_BYTES % 1024 == 0, "staging must stay 1024-byte aligned");
  static_assert(!KS || part_bytes<BN>() <= STAGES * (A_BYTES + B_BYTES), "split-K send buffer larger than the pipeline stages");
  pdl_trigger();
  if ((KS && S > 1 && (int)(gridDim.x / S) < args.ntiles) || (QB && (int)gridDim.x < args.ntiles * S)) {  // one unit per cluster / CTA
    pdl_wait();
    if (threadIdx.x == 0) atomicOr(&g_gemm_err, 2u);
    return;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int r = 0; r < EPI_WARPS; r++) mbar_init(&rbar[r], 1);
    for (int a = 0; a < 2; a++) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], EPI_WARPS);
    }
    mbar_init(&pbar[0], 1);
    if (KS && S > 1) mbar_arrive_expect_tx(&pbar[0], part_bytes<BN>());  // S slots of 128/S rows
    if (QB)
      for (int s = 0; s < STAGES; s++) {
        mbar_init(&pfull[s], 1);
        mbar_init(&conv[s], EPI_WARPS);
      }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmA) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmB) : "memory");
  }
  if constexpr (KS) cluster_sync();  // every CTA's barriers exist before a remote arrival
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // A weight no kernel of the chain writes is requested before the
  // dependency wait: the first tile's first STAGES weight blocks go to their
  // stages (whose barriers then expect the activation block as well) and the
  // rest of its K range into L2.
  int pre = 0;
  int issued[STAGES], pk_issued[STAGES];
  uint32_t iss_phase[STAGES], pk_phase[STAGES];
  for (int s = 0; s < STAGES; s++) issued[s] = 0, iss_phase[s] = 0, pk_issued[s] = 0, pk_phase[s] = 0;
  const int pkb = QB ? BK * args.q.bits / 8 : 0;  // packed bytes per row of a block
  if (QB && warp == 0 && lane == 0 && (int)blockIdx.x < args.ntiles * S) {
    const int w = blockIdx.x, t = w / S, kb0 = (w % S) * KB / S, kb1 = (w % S + 1) * KB / S;
    const int n0 = (t % args.ntile_n) * BN;
    for (int kb = kb0; kb < kb1 && pre < STAGES; kb++) {
      mbar_arrive_expect_tx(&pfull[pre], (uint32_t)(BN * pkb));
      tma_load_2d(sPk + pre * PK_BYTES, &tmB, &pfull[pre], kb * pkb, n0);
      pk_issued[pre++] = 1;
    }
  } else if (!QB && warp == 0 && lane == 0 && args.ep.w_static && (int)blockIdx.x < args.ntiles * S) {
    const int w = blockIdx.x, t = w / S, kb0 = (w % S) * KB / S, kb1 = (w % S + 1) * KB / S;
    const int n0 = (t % args.ntile_n) * BN;
    for (int kb = kb0; kb < kb1; kb++) {
      if (pre < STAGES) {
        mbar_arrive_expect_tx(&full[pre], A_BYTES + B_BYTES);
        tma_load_2d(sB + pre * B_BYTES, &tmB, &full[pre], kb * BK, n0);
        issued[pre++] = 1;
      } else {
        tma_prefetch_l2(&tmB, kb * BK, n0);
      }
    }
  }
  if (warp == 0 && lane == 0 && args.ep.l2_next) {  // this CTA's slice of the next projection's weight
    const size_t total = args.ep.l2_next_bytes & ~(size_t)15;
    const size_t per = ((total + gridDim.x - 1) / gridDim.x + 15) & ~(size_t)15;
    const size_t lo = per * blockIdx.x, hi = lo + per < total ? lo + per : total;
    for (size_t o = lo; o < hi; o += 65536) bulk_prefetch_l2((const char*)args.ep.l2_next + o, (uint32_t)(hi - o < 65536 ? hi - o : 65536));
  }
  if (!QB) pdl_wait();  // the kernel that wrote the activations has completed

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      if (QB) pdl_wait();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;  // k blocks issued so far (the first `pre` have their weight block in flight)
      for (int w = blockIdx.x; w < args.ntiles * S && ok; w += gridDim.x) {
        const int t = w / S, kb0 = (w % S) * KB / S, kb1 = (w % S + 1) * KB / S;
        int m0 = (t / args.ntile_n) * BM, n0 = (t % args.ntile_n) * BN;
        for (int kb = kb0; kb < kb1; kb++, it++) {
          if (QB) {
            if (!mbar_wait(&empty[stage], phase ^ 1, abort, &g_gemm_err)) { ok = false; break; }
            mbar_arrive_expect_tx(&full[stage], A_BYTES);
            tma_load_2d(sA + stage * A_BYTES, &tmA, &full[stage], kb * BK, m0);
            if (it >= pre) {
              mbar_arrive_expect_tx(&pfull[stage], (uint32_t)(BN * pkb));
              tma_load_2d(sPk + stage * PK_BYTES, &tmB, &pfull[stage], kb * pkb, n0);
              pk_issued[stage] = 1;
              pk_phase[stage] = phase;
            }
          } else if (it < pre) {
            tma_load_2d(sA + stage * A_BYTES, &tmA, &full[stage], kb * BK, m0);
          } else {
            if (!mbar_wait(&empty[stage], phase ^ 1, abort, &g_gemm_err)) { ok = false; break; }
            mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
            tma_load_2d(sA + stage * A_BYTES, &tmA, &full[stage], kb * BK, m0);
            tma_load_2d(sB + stage * B_BYTES, &tmB, &full[stage], kb * BK, n0);
          }
          issued[stage] = 1;
          iss_phase[stage] = phase;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // drain: every copy this thread issued must have landed before the CTA exits
      for (int s = 0; s < STAGES; s++) {
        if (issued[s]) {
          uint64_t t0 = gtimer();
          while (!mbar_try_wait(&full[s], iss_phase[s]) && gtimer() - t0 < kWaitNs) {}
        }
        if (QB && pk_issued[s]) {
          uint64_t t0 = gtimer();
          while (!mbar_try_wait(&pfull[s], pk_phase[s]) && gtimer() - t0 < kWaitNs) {}
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16<T, BN>();
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool committed = false;
      uint64_t* last = nullptr;
      uint32_t last_phase = 0;
      for (int w = blockIdx.x; w < args.ntiles * S && ok; w += gridDim.x) {
        const int kb0 = (w % S) * KB / S, kb1 = (w % S + 1) * KB / S;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort, &g_gemm_err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int kb = kb0; kb < kb1; kb++) {
          if (!mbar_wait(&full[stage], phase, abort, &g_gemm_err)) { ok = false; break; }
          if (QB && !mbar_wait(&conv[stage], phase, abort, &g_gemm_err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES), b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; k++)
            tc_mma(d, sdesc_sw128(a0 + k * 32), sdesc_sw128(b0 + k * 32), idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          tc_commit(&empty[stage]);
          committed = true;
          last = &empty[stage];
          last_phase = phase;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      // drain: the MMAs this thread issued must finish before TMEM is freed
      if (committed) {
        uint64_t t0 = gtimer();
        while (!mbar_try_wait(last, last_phase) && gtimer() - t0 < kWaitNs) {}
      }
    }
  } else if constexpr (TMAE) {
    if constexpr (QB) {  // dequantise the packed blocks as they land, then wait for the predecessor
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < args.ntiles * S && ok; w += gridDim.x) {
        const int t = w / S, kb0 = (w % S) * KB / S, kb1 = (w % S + 1) * KB / S;
        const int n0 = (t % args.ntile_n) * BN;
        for (int kb = kb0; kb < kb1; kb++) {
          float2 sbv[conv_tasks<BN>()];
          load_packed_scales<BN>(args, n0, kb, (int)threadIdx.x - 64, sbv);  // in flight while the block lands
          if (!mbar_wait(&pfull[stage], phase, abort, &g_gemm_err)) { ok = false; break; }
          convert_packed_block<T, BN>(args, sPk + stage * PK_BYTES, sB + stage * B_BYTES, n0, kb, (int)threadIdx.x - 64, sbv);
          fence_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&conv[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      pdl_wait();  // the kernel that wrote the activations and the residual has completed
    }
    if (KS && S > 1)
      epilogue_split<T, BN, EPI_WARPS>(args, &tmY, sE, tfull, tempty, abort, tmem, warp, lane, sP, (float*)sA, pbar);
    else
      epilogue_tma<T, BN, false, EPI_WARPS, 1, KS>(args, &tmY, &tmR, sE, rbar, tfull, tempty, abort, tmem, warp, lane, blockIdx.x / S,
                                                   gridDim.x / S, BM, 0, sP, (float*)sA, pbar);
  } else {
    // ---------------- epilogue (warps 2..9 -> TMEM lane quarter warp % 4, half of the units each)
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    constexpr int U = BN / 64;
    const bool vec = args.vec_ok != 0;
    T* Y = (T*)args.y;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < args.ntiles; t += gridDim.x) {
      if (!mbar_wait(&tfull[acc], acc_phase, abort, &g_gemm_err)) break;
      tc_fence_after();
      const int m0 = (t / args.ntile_n) * BM, n0 = (t % args.ntile_n) * BN;
      const int row = m0 + quarter * 32 + lane;
      const bool live = row < args.M;
      T* rowp = Y + (int64_t)row * args.ldy;
      const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
      float ln_mu, ln_r;
      if (args.ep.ln_stats) ln_row(args.ep, row, args.M, ln_mu, ln_r);
#pragma unroll 1
      for (int u = half * (U / 2); u < (half + 1) * (U / 2); u++) {
        uint32_t ra[32], rb[32];
        tmem_ld32(tbase + u * 64, ra);
        tmem_ld32(tbase + u * 64 + 32, rb);
        tmem_wait_ld();
        float a[32], b[32];
#pragma unroll
        for (int j = 0; j < 32; j++) a[j] = __uint_as_float(ra[j]), b[j] = __uint_as_float(rb[j]);
        const int col = n0 + u * 64;
        if (!live || col >= (args.ep.kind == EPI_GEGLU ? 2 * args.N : args.N)) continue;
        const GemmEpilogue& ep = args.ep;
        if (ep.ln_stats) ln_apply(ep, col, ln_mu, ln_r, a, b);
        if (ep.kind == EPI_GEGLU) {
#pragma unroll
          for (int j = 0; j < 32; j++) a[j] = gelu_exact(a[j]) * b[j];
          store32<T>(rowp, col / 2, args.N, a, vec);
          continue;
        }
        if (ep.kind == EPI_ROPE_QKV && col < ep.rope_cols) {
          const float4* rq = (const float4*)ep.rope_cs + ep.pos[row];
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const float4 v = __ldg(rq + (int64_t)(j >> 1) * ep.rope_cap);
            const float c = (j & 1) ? v.y : v.x, sn = (j & 1) ? v.w : v.z;
            const float x1 = a[j], x2 = b[j];
            a[j] = x1 * c - x2 * sn;
            b[j] = x2 * c + x1 * sn;
          }
        }
        if (args.bias) {
#pragma unroll
          for (int j = 0; j < 32; j++) {
            if (col + j < args.N) a[j] += ld_as<float>((const char*)args.bias, args.bias_dtype, col + j);
            if (col + 32 + j < args.N) b[j] += ld_as<float>((const char*)args.bias, args.bias_dtype, col + 32 + j);
          }
        }
        if (ep.kind == EPI_RESIDUAL) {
          const T* rp = (const T*)ep.resid + (int64_t)row * ep.ldr;
          float r[32];
          load32f<T>(rp, col, args.N, r, vec);
#pragma unroll
          for (int j = 0; j < 32; j++) a[j] += r[j];
          load32f<T>(rp, col + 32, args.N, r, vec);
#pragma unroll
          for (int j = 0; j < 32; j++) b[j] += r[j];
          if (ep.stats_out) ep.stats_out[(int64_t)row * (args.N / 64) + col / 64] = stats_unit<T>(a, b);
        }
        store32<T>(rowp, col, args.N, a, vec);
        store32<T>(rowp, col + 32, args.N, b, vec);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }
  if (threadIdx.x == 0 && *abort) {  // after a timeout, let copies still in flight land before the CTA exits
    const uint64_t t0 = gtimer();
    while (gtimer() - t0 < 1000000ull) {}
  }
  tc_fence_before();
  if constexpr (KS) cluster_sync();  // no CTA leaves while another may read its partial or arrive on its barriers
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}


// CTA-pair GEMM (cluster of two CTAs, tcgen05 cta_group::2): a pair computes a
// 256 x 256 output tile. Each CTA loads its 128 rows of x and its 128 of the
// tile's 256 rows of w per 64-wide k-step (32 KB, half the weight bytes per
// CTA of the single-CTA kernel) and keeps its 128 x 256 accumulator in its
// own TMEM. The thread of CTA 0 issues the M = 256 MMAs for both; the loads
// of both CTAs complete on CTA 0's full barrier, and every MMA commit arrives
// on the empty / accumulator-full barriers of both CTAs. The epilogue is the
// single-CTA one on each CTA's rows. No load is multicast.
template <int STAGES>
constexpr size_t gemm_pair_smem_bytes() {
  return (size_t)STAGES * (BM * BK * 2 + 128 * BK * 2) + PAIR_EPI_WARPS * PAIR_NBUF * 4096 + 1024 + 512;
}

template <typename T, int STAGES>
__global__ void __launch_bounds__(PAIR_THREADS, 1) k_gemm_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                                                           const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmR,
                                                           const __grid_constant__ GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  constexpr int BN = 256;
  constexpr uint32_t A_BYTES = BM * BK * 2;
  constexpr uint32_t B_BYTES = 128 * BK * 2;  // this CTA's half of the tile's w rows
  constexpr uint32_t TMEM_COLS = 2 * BN;
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sE = sB + STAGES * B_BYTES;                                  // PAIR_NBUF staging buffers per epilogue warp
  uint64_t* full = (uint64_t*)(sE + PAIR_EPI_WARPS * PAIR_NBUF * 4096);  // used in CTA 0
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;  // used in CTA 0: both CTAs' epilogue warps arrive
  uint64_t* rbar = tempty + 2;   // one per staging buffer
  uint32_t* tmem_slot = (uint32_t*)(rbar + PAIR_EPI_WARPS * PAIR_NBUF);
  volatile int* abort = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = (args.K + BK - 1) / BK;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int r = 0; r < PAIR_EPI_WARPS * PAIR_NBUF; r++) mbar_init(&rbar[r], 1);
    for (int a = 0; a < 2; a++) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * PAIR_EPI_WARPS);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {  // the same warp of both CTAs: one allocation at the same TMEM address in each
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmA) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmB) : "memory");
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before any remote arrival or copy
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // the kernel that wrote the activations has completed

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs)
    if (lane == 0) {
      const uint32_t full0 = mapa_rank(smem_u32(full), 0);  // CTA 0's full[0]
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int issued[STAGES];
      uint32_t iss_phase[STAGES];
      for (int s = 0; s < STAGES; s++) issued[s] = 0, iss_phase[s] = 0;
      for (int t = pair; t < args.ntiles && ok; t += npairs) {
        const int m0 = (t / args.ntile_n) * (2 * BM) + rank * BM, n0 = (t % args.ntile_n) * BN + rank * 128;
        for (int kb = 0; kb < KB; kb++) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort, &g_gemm_err)) { ok = false; break; }
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (A_BYTES + B_BYTES));
          tma_load_2d_pair(sA + stage * A_BYTES, &tmA, full0 + 8 * stage, kb * BK, m0);
          tma_load_2d_pair(sB + stage * B_BYTES, &tmB, full0 + 8 * stage, kb * BK, n0);
          issued[stage] = 1;
          iss_phase[stage] = phase;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // drain: each stage's last fill has been consumed by the pair's MMAs (so it landed)
      for (int s = 0; s < STAGES; s++)
        if (issued[s]) {
          uint64_t t0 = gtimer();
          bool done;
          while (!(done = mbar_try_wait(&empty[s], iss_phase[s])) && gtimer() - t0 < kWaitNs) {}
          if (!done) *abort = 1;
        }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (CTA 0 only)
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = idesc_f16<T, BN, 256>();
      const uint64_t dA0 = sdesc_sw128(smem_u32(sA)), dB0 = sdesc_sw128(smem_u32(sB));
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      uint64_t* last = nullptr;
      uint32_t last_phase = 0;
      for (int t = pair; t < args.ntiles && ok; t += npairs) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort, &g_gemm_err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int kb = 0; kb < KB; kb++) {
          if (!mbar_wait(&full[stage], phase, abort, &g_gemm_err)) { ok = false; break; }
          tc_fence_after();
          const uint64_t da = dA0 + ((stage * A_BYTES) >> 4), db = dB0 + ((stage * B_BYTES) >> 4);
#pragma unroll
          for (int k = 0; k < BK / 16; k++) tc_mma_pair(d, da + k * 2, db + k * 2, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          tc_commit_pair(&empty[stage]);
          last = &empty[stage];
          last_phase = phase;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit_pair(&tfull[acc]);
        last = &tfull[acc];
        last_phase = acc_phase;
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      // drain: the MMAs issued here finish before TMEM is freed
      if (last) {
        uint64_t t0 = gtimer();
        while (!mbar_try_wait(last, last_phase) && gtimer() - t0 < kWaitNs) {}
      }
    }
  } else {
    epilogue_tma<T, BN, true, PAIR_EPI_WARPS, PAIR_NBUF>(args, &tmY, &tmR, sE, rbar, tfull, tempty, abort, tmem, warp, lane, pair, npairs, 2 * BM,
                                                 (int)rank * BM);
  }
  if (threadIdx.x == 0 && *abort) {  // after a timeout, let copies still in flight land before the pair exits
    const uint64_t t0 = gtimer();
    while (gtimer() - t0 < 1000000ull) {}
  }
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its partner may still read its shared memory or arrive on its barriers
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    CUDA_OK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    LC_CHECK(q == cudaDriverEntryPointSuccess && p, "cuTensorMapEncodeTiled is not available from the driver");
    fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  }
  return fn;
}

using MapKey = std::tuple<uintptr_t, int64_t, int64_t, int64_t, int, int>;
std::map<MapKey, CUtensorMap>& map_cache() {
  static std::map<MapKey, CUtensorMap> m;
  return m;
}

// Row-major [rows, K] matrix, boxes of box_rows x 64, 128-byte swizzle.
// Row-major [rows, cols] matrix with row stride ld (elements), boxes of
// box_rows x box_cols (box_cols * 2 bytes = 128: one swizzle row).
// Returned by value: a later call may clear the cache.
CUtensorMap tensor_map(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_cols, int box_rows, int dtype) {
  MapKey key{(uintptr_t)ptr, rows, cols, ld, box_cols * 1024 + box_rows, dtype};
  auto& c = map_cache();
  auto it = c.find(key);
  if (it != c.end()) return it->second;
  if (c.size() > 8192) c.clear();
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = encode_fn()(&m, dtype == LC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr),
                           dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LC_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return c.emplace(key, m).first->second;
}
// Bytes of a row-major [rows, cols] byte matrix (the packed weights), boxes of
// box_rows x box_cols bytes, no swizzle.
CUtensorMap tensor_map_u8(const void* ptr, int64_t rows, int64_t cols, int box_cols, int box_rows) {
  MapKey key{(uintptr_t)ptr, rows, cols, cols, box_cols * 1024 + box_rows, -1};
  auto& c = map_cache();
  auto it = c.find(key);
  if (it != c.end()) return it->second;
  if (c.size() > 8192) c.clear();
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LC_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return c.emplace(key, m).first->second;
}

template <typename T, int BN, int STAGES, bool TMAE>
void launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& my, const CUtensorMap& mr, const GemmArgs& a,
                 cudaStream_t st) {
  constexpr size_t smem = gemm_smem_bytes<STAGES, BN>(TMAE);
  static_assert(smem <= 232448, "GEMM shared memory above the 227 KB per-CTA limit");
  static bool attr = false;
  if (!attr) {
    CUDA_OK(cudaFuncSetAttribute(k_gemm_tc<T, BN, STAGES, TMAE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr = true;
  }
  int grid = std::min(a.ntiles, lc::num_sms());
  lc::launch_chain(k_gemm_tc<T, BN, STAGES, TMAE>, dim3(grid), dim3(GEMM_THREADS), smem, st, ma, mb, my, mr, a);
}

// Split K: clusters of a.ksplit CTAs, one cluster per tile while they fit
// (QB: the packed-weight instance).
template <typename T, int BN, int STAGES, bool QB = false>
cudaLaunchConfig_t split_config(int S, cudaLaunchAttribute* at, cudaStream_t st) {
  constexpr size_t smem = gemm_smem_bytes<STAGES, BN>(true, true, QB);
  static_assert(smem <= 232448, "GEMM shared memory above the 227 KB per-CTA limit");
  static bool attr = false;
  if (!attr) {
    CUDA_OK(cudaFuncSetAttribute(k_gemm_tc<T, BN, STAGES, true, true, QB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = S;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  lc::chain_attrs(cfg, at, 1);
  return cfg;
}
// clusters of S of this instance that can be resident at once
template <typename T, int BN, int STAGES, bool QB = false>
int split_capacity(int S) {
  static int cap[5] = {0, 0, 0, 0, 0};
  if (!cap[S]) {
    cudaLaunchAttribute at[2];
    cudaLaunchConfig_t cfg = split_config<T, BN, STAGES, QB>(S, at, nullptr);
    cfg.gridDim = dim3(S * (lc::num_sms() / S));
    int n = 0;
    CUDA_OK(cudaOccupancyMaxActiveClusters(&n, k_gemm_tc<T, BN, STAGES, true, true, QB>, &cfg));
    LC_CHECK(n > 0, "tcgen05 GEMM: no split-K cluster fits");
    cap[S] = n;
  }
  return cap[S];
}
template <typename T, int BN, int STAGES, bool QB = false>
void launch_gemm_split(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& my, const CUtensorMap& mr, const GemmArgs& a,
                       cudaStream_t st) {
  const int S = a.ksplit;
  LC_CHECK(S == 1 || S == 2 || S == 4, "tcgen05 GEMM: split-K factor must be 1, 2 or 4");
  cudaLaunchAttribute at[2];
  cudaLaunchConfig_t cfg = split_config<T, BN, STAGES, QB>(S, at, st);
  const int cap = split_capacity<T, BN, STAGES, QB>(S);
  LC_CHECK((S == 1 && !QB) || a.ntiles <= cap, "tcgen05 GEMM: split K needs one resident cluster per tile");
  cfg.gridDim = dim3(S * std::min(a.ntiles, cap));
  CUDA_OK(cudaLaunchKernelEx(&cfg, k_gemm_tc<T, BN, STAGES, true, true, QB>, ma, mb, my, mr, a));
}
int split_capacity_for(int dtype, int BN, int S, bool qb = false) {
  if (qb) {
    if (dtype == LC_F16) return BN == 64 ? split_capacity<__half, 64, 4, true>(S) : split_capacity<__half, 128, 3, true>(S);
    return BN == 64 ? split_capacity<__nv_bfloat16, 64, 4, true>(S) : split_capacity<__nv_bfloat16, 128, 3, true>(S);
  }
  if (dtype == LC_F16) return BN == 64 ? split_capacity<__half, 64, 4>(S) : split_capacity<__half, 128, 3>(S);
  return BN == 64 ? split_capacity<__nv_bfloat16, 64, 4>(S) : split_capacity<__nv_bfloat16, 128, 3>(S);
}

template <typename T, int STAGES>
void launch_gemm_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& my, const CUtensorMap& mr, GemmArgs a, cudaStream_t st) {
  constexpr size_t smem = gemm_pair_smem_bytes<STAGES>();
  static_assert(smem <= 232448, "GEMM shared memory above the 227 KB per-CTA limit");
  static int max_pairs = 0;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(PAIR_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  lc::chain_attrs(cfg, at, 1);
  if (!max_pairs) {
    CUDA_OK(cudaFuncSetAttribute(k_gemm_pair<T, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cfg.gridDim = dim3(2 * (lc::num_sms() / 2));
    int n = 0;
    CUDA_OK(cudaOccupancyMaxActiveClusters(&n, k_gemm_pair<T, STAGES>, &cfg));
    LC_CHECK(n > 0, "tcgen05 GEMM: no CTA pair fits an SM pair");
    max_pairs = n;
  }
  const int pairs = std::min(a.ntiles, max_pairs);
  cfg.gridDim = dim3(2 * pairs);
  CUDA_OK(cudaLaunchKernelEx(&cfg, k_gemm_pair<T, STAGES>, ma, mb, my, mr, a));
}

}  // namespace

namespace lc {

// 256-wide tiles run on CTA pairs (half the weight bytes per CTA, two staging
// buffers per epilogue warp); LAYA_CUDA_GEMM_PAIR=0 selects the single-CTA
// kernel instead (both are tested).
bool gemm_use_pair(int64_t K) {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("LAYA_CUDA_GEMM_PAIR");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  (void)K;
  return on == 1;
}

// Small-M launches use narrow tiles with K split over clusters;
// LAYA_CUDA_GEMM_SPLIT=0 keeps them on the ordinary tiles (both are tested).
bool gemm_use_split() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("LAYA_CUDA_GEMM_SPLIT");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

bool gemm_raw(const void* x, int64_t M, int64_t K, const void* w, int64_t N, const void* bias, int bias_dtype, void* y, int64_t ldy,
              int dtype, const GemmEpilogue& ep, cudaStream_t st) {
  if (!(dtype == LC_F16 || dtype == LC_BF16)) return false;
  if (M <= 0 || N <= 0 || K < 16 || K % 8) return false;
  if (((uintptr_t)x | (uintptr_t)w) & 15) return false;
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return false;
  // the accumulator width covered by the weight rows: GeGLU produces N outputs from 2N rows
  int64_t Nacc = ep.kind == EPI_GEGLU ? 2 * N : N;
  const int BN = gemm_tile_n(Nacc, ep.kind == EPI_GEGLU);
  if (ep.kind == EPI_ROPE_QKV && (ep.rope_cols % 64)) return false;
  // folded-LayerNorm statistics cover whole 64-column units
  if (ep.stats_out && (ep.kind != EPI_RESIDUAL || N % 64)) return false;
  if (ep.ln_stats && (Nacc % 64 || ((uintptr_t)ep.ln_wsum & 15) || ep.ln_parts < 1 || ep.ln_parts > LN_MAX_PARTS ||
                      (int64_t)ep.ln_parts * ep.ln_part_cols < K || ep.ln_cols != K))
    return false;
  GemmArgs a{};
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.ntile_n = (int)((Nacc + BN - 1) / BN);
  int64_t tiles = ((M + BM - 1) / BM) * a.ntile_n;
  if (tiles > INT32_MAX) return false;
  a.ntiles = (int)tiles;
  a.y = y;
  a.ldy = ldy;
  a.vec_ok = (ldy % 8 == 0 && ((uintptr_t)y & 15) == 0 && (ep.kind != EPI_RESIDUAL || (ep.ldr % 8 == 0 && ((uintptr_t)ep.resid & 15) == 0))) ? 1 : 0;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.ep = ep;
  a.ksplit = 1;
  const CUtensorMap& ma = tensor_map(x, M, K, K, BK, BM, dtype);
  const CUtensorMap& mb = tensor_map(w, Nacc, K, K, BK, BN, dtype);
  // TMA-store epilogue when the output (and residual) rows are 16-byte strided and aligned
  const bool tmae = a.vec_ok && (N % 8 == 0) && !(ep.kind == EPI_RESIDUAL && ep.resid == nullptr);
  const int sms = lc::num_sms();
  if (tmae && gemm_use_split() && tiles * 4 <= sms) {
    // Few rows (one prompt, a small batch): the natural tiles would occupy a
    // few SMs, each bound by its own tensor pipe. Narrow tiles (64 columns,
    // 128 for GeGLU's gate/up pairs) and K split over clusters of up to 4 CTAs
    // spread the weight stream and the MMAs over most of the GPU.
    const int BNs = ep.kind == EPI_GEGLU ? 128 : 64;
    const int64_t mt = (M + BM - 1) / BM, nt = (Nacc + BNs - 1) / BNs;
    const int KB = (int)((K + BK - 1) / BK);
    int S = 1;
    for (int c : {4, 2})
      if (mt * nt * c <= sms && KB >= c && mt * nt <= split_capacity_for(dtype, BNs, c)) {
        S = c;
        break;
      }
    GemmArgs as = a;
    as.ntile_n = (int)nt;
    as.ntiles = (int)(mt * nt);
    as.ksplit = S;
    const CUtensorMap& mbs = tensor_map(w, Nacc, K, K, BK, BNs, dtype);
    // split: the owner's warps store R rows at a time (epilogue_split)
    const CUtensorMap& my = tensor_map(y, M, N, ldy, 64, S > 1 ? (BNs == 128 ? 2 : 4) : 32, dtype);
    const CUtensorMap& mr = ep.kind == EPI_RESIDUAL ? tensor_map(ep.resid, M, N, ep.ldr, 64, 32, dtype) : my;
    if (dtype == LC_F16) {
      if (BNs == 64) launch_gemm_split<__half, 64, 4>(ma, mbs, my, mr, as, st);
      else launch_gemm_split<__half, 128, 3>(ma, mbs, my, mr, as, st);
    } else {
      if (BNs == 64) launch_gemm_split<__nv_bfloat16, 64, 4>(ma, mbs, my, mr, as, st);
      else launch_gemm_split<__nv_bfloat16, 128, 3>(ma, mbs, my, mr, as, st);
    }
  } else if (tmae && BN == 256 && gemm_use_pair(K)) {
    // CTA pairs: 256 x 256 tiles
    const CUtensorMap& my = tensor_map(y, M, N, ldy, 64, 32, dtype);
    const CUtensorMap& mr = ep.kind == EPI_RESIDUAL ? tensor_map(ep.resid, M, N, ep.ldr, 64, 32, dtype) : my;
    const CUtensorMap& mbp = tensor_map(w, Nacc, K, K, BK, 128, dtype);
    GemmArgs ap = a;
    const int64_t ptiles = ((M + 2 * BM - 1) / (2 * BM)) * a.ntile_n;
    ap.ntiles = (int)ptiles;
    if (dtype == LC_F16) launch_gemm_pair<__half, 5>(ma, mbp, my, mr, ap, st);
    else launch_gemm_pair<__nv_bfloat16, 5>(ma, mbp, my, mr, ap, st);
  } else if (tmae) {
    const CUtensorMap& my = tensor_map(y, M, N, ldy, 64, 32, dtype);
    const CUtensorMap& mr = ep.kind == EPI_RESIDUAL ? tensor_map(ep.resid, M, N, ep.ldr, 64, 32, dtype) : my;
    if (dtype == LC_F16) {
      if (BN == 256) launch_gemm<__half, 256, 4, true>(ma, mb, my, mr, a, st);
      else launch_gemm<__half, 128, 6, true>(ma, mb, my, mr, a, st);
    } else {
      if (BN == 256) launch_gemm<__nv_bfloat16, 256, 4, true>(ma, mb, my, mr, a, st);
      else launch_gemm<__nv_bfloat16, 128, 6, true>(ma, mb, my, mr, a, st);
    }
  } else {
    if (dtype == LC_F16) {
      if (BN == 256) launch_gemm<__half, 256, 4, false>(ma, mb, ma, ma, a, st);
      else launch_gemm<__half, 128, 6, false>(ma, mb, ma, ma, a, st);
    } else {
      if (BN == 256) launch_gemm<__nv_bfloat16, 256, 4, false>(ma, mb, ma, ma, a, st);
      else launch_gemm<__nv_bfloat16, 128, 6, false>(ma, mb, ma, ma, a, st);
    }
  }
  LC_LAUNCHED(1);
  return true;
}

// In-kernel dequantisation for few rows; LAYA_CUDA_QGEMM_FUSED=0 makes
// gemm_raw_q decline (the caller then dequantises into a dense scratch).
bool gemm_use_qfused() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("LAYA_CUDA_QGEMM_FUSED");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

bool gemm_raw_q(const void* x, int64_t M, int64_t K, const GemmQuantB& q, int64_t N, const void* bias, int bias_dtype, void* y,
                int64_t ldy, int dtype, const GemmEpilogue& ep, cudaStream_t st) {
  if (!gemm_use_qfused()) return false;
  if (!(dtype == LC_F16 || dtype == LC_BF16)) return false;
  if (!(q.bits == 4 || q.bits == 8) || q.group < 8 || q.group % 8 || !q.w || !q.scales) return false;
  if (M <= 0 || N <= 0 || K < BK || K % 8) return false;
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return false;
  const int64_t rowb = K * q.bits / 8;  // packed bytes per weight row
  if (rowb % 16 || (((uintptr_t)q.w | (uintptr_t)x | (uintptr_t)q.gamma) & 15)) return false;
  const bool geglu = ep.kind == EPI_GEGLU;
  const int64_t Nacc = geglu ? 2 * N : N;
  if (ep.kind == EPI_ROPE_QKV && (ep.rope_cols % 64)) return false;
  if (ep.stats_out && (ep.kind != EPI_RESIDUAL || N % 64)) return false;
  if (ep.ln_stats && (Nacc % 64 || ((uintptr_t)ep.ln_wsum & 15) || ep.ln_parts < 1 || ep.ln_parts > LN_MAX_PARTS ||
                      (int64_t)ep.ln_parts * ep.ln_part_cols < K || ep.ln_cols != K))
    return false;
  const bool vec_ok = ldy % 8 == 0 && ((uintptr_t)y & 15) == 0 && (ep.kind != EPI_RESIDUAL || (ep.ldr % 8 == 0 && ((uintptr_t)ep.resid & 15) == 0));
  if (!vec_ok || N % 8 || (ep.kind == EPI_RESIDUAL && !ep.resid)) return false;
  // few rows only: the natural tiles would fill at most a quarter of the SMs
  const int sms = lc::num_sms();
  const int64_t mt = (M + BM - 1) / BM;
  const int BN0 = gemm_tile_n(Nacc, geglu);
  if (mt * ((Nacc + BN0 - 1) / BN0) * 4 > sms) return false;
  const int BNs = geglu ? 128 : 64;
  const int64_t nt = (Nacc + BNs - 1) / BNs;
  const int KB = (int)((K + BK - 1) / BK);
  int S = 0;
  for (int c : {4, 2, 1})
    if (mt * nt * c <= sms && KB >= c && mt * nt <= split_capacity_for(dtype, BNs, c, true)) {
      S = c;
      break;
    }
  if (!S) return false;
  GemmArgs a{};
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.ntile_n = (int)nt;
  a.ntiles = (int)(mt * nt);
  a.y = y;
  a.ldy = ldy;
  a.vec_ok = 1;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.ep = ep;
  a.ksplit = S;
  a.q = q;
  const CUtensorMap& ma = tensor_map(x, M, K, K, BK, BM, dtype);
  const CUtensorMap& mb = tensor_map_u8(q.w, Nacc, rowb, BK * q.bits / 8, BNs);
  const CUtensorMap& my = tensor_map(y, M, N, ldy, 64, S > 1 ? (BNs == 128 ? 2 : 4) : 32, dtype);
  const CUtensorMap& mr = ep.kind == EPI_RESIDUAL ? tensor_map(ep.resid, M, N, ep.ldr, 64, 32, dtype) : my;
  if (dtype == LC_F16) {
    if (BNs == 64) launch_gemm_split<__half, 64, 4, true>(ma, mb, my, mr, a, st);
    else launch_gemm_split<__half, 128, 3, true>(ma, mb, my, mr, a, st);
  } else {
    if (BNs == 64) launch_gemm_split<__nv_bfloat16, 64, 4, true>(ma, mb, my, mr, a, st);
    else launch_gemm_split<__nv_bfloat16, 128, 3, true>(ma, mb, my, mr, a, st);
  }
  LC_LAUNCHED(1);
  return true;
}

// GeGLU needs whole (gate, up) 64-column unit pairs in every tile that holds
// data: Nacc % 128 == 0 is enough for 256-wide tiles (a last tile of 128
// columns leaves its second half empty; configs[4]'s 2 x 2624 = 5248).
int gemm_tile_n(int64_t Nacc, bool geglu) {
  int BN = (Nacc % 256 == 0 || Nacc > 1024) ? 256 : 128;
  if (geglu && Nacc % 128) BN = 128;
  return BN;
}

int gemm_stats_part_cols(int64_t N) {
  (void)N;
  return 64;
}

bool gemm_linear(const LcTensor* x2, const LcTensor* w, const LcTensor* bias, LcTensor* y, const GemmEpilogue& ep) {
  int64_t M = x2->shape[0], K = x2->shape[1], N = w->shape[0];
  if (K < 64) return false;  // tiny reductions stay on the SIMT path
  return gemm_raw(x2->data(), M, K, w->data(), N, bias ? bias->data() : nullptr, bias ? bias->dtype : 0, y->data(), N, y->dtype, ep,
                  stream());
}

std::string take_device_errors() {
  unsigned int e = 0, z = 0;
  CUDA_OK(cudaMemcpyFromSymbol(&e, g_gemm_err, sizeof(e)));
  std::string msg = take_attention_errors();
  if (!e) return msg;
  CUDA_OK(cudaMemcpyToSymbol(g_gemm_err, &z, sizeof(z)));
  std::string what = (e & 1u) ? "a pipeline wait timed out (kernel aborted its tile loop)" : "a split-K launch had more tiles than clusters";
  return "tcgen05 GEMM: " + what + (msg.empty() ? std::string() : "; " + msg);
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() { return encode_fn(); }

CUtensorMap tensor_map_2d(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_cols, int box_rows, int dtype) {
  return tensor_map(ptr, rows, cols, ld, box_cols, box_rows, dtype);
}

}  // namespace lc

void lc_gemm_destroy_caches() { map_cache().clear(); }

// Sets this unit's bounded-wait limit (lc_debug_set_wait_limit).
void lc_internal_wait_limit_gemm(unsigned long long ns) { CUDA_OK(cudaMemcpyToSymbol(sm100::g_wait_limit_ns, &ns, sizeof(ns))); }

// A kernel whose one wait nothing satisfies: it gives up after the bounded
// wait's limit, records the timeout in the GEMM error word and returns, so
// the host sees the error at its next lc_flush / lc_read while the context
// stays usable. Only lc_debug_stuck_wait launches it.
__global__ void k_wait_probe() {
  __shared__ uint64_t bar;
  __shared__ int abort;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);
    abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) sm100::mbar_wait(&bar, 0, (volatile int*)&abort, &g_gemm_err);
}

void lc_internal_launch_wait_probe() {
  k_wait_probe<<<1, 32, 0, lc::stream()>>>();
  LC_LAUNCHED(1);
}
