// Tensor-core (tcgen05 / TMEM) flash attention over unpadded varlen sequences,
// head dim 64 — the attention of ModernBert.layer
// (packages/modernbert/src/index.ts:348-352: sdpa with the masks of
// attentionMasks, index.ts:240-259) computed without masks or padding.
//
// Persistent: two CTAs per SM, each walking the work list (128-query-row tile
// of one sequence x head; tiles longest sequence first) with a stride of the
// grid. Key blocks of 64. Roles:
//   warp 0      TMA producer: Q of each work item into one of two Q buffers
//               (the next item's Q loads while the current one runs), K and V
//               blocks into an NST-stage ring that runs on across items
//               (128 x 64 / 64 x 64 tiles of the fused [T, 3H] projection,
//               128-byte swizzle);
//   warp 1      TMEM owner and single-thread MMA issuer:
//                 S_j = Q·K_jᵀ  (M=128, N=64, K=64; A, B from shared memory)
//                 O  += P_j·V_j (M=128, N=64, K=64; A = P from TMEM, B = V
//                                from shared memory, MN-major)
//               S is double-buffered in TMEM (columns 0-63 / 64-127), so
//               S_{j+1} runs while the softmax works on S_j, also across work
//               items; O is double-buffered by work-item parity (columns
//               128-191 / 192-255; 256 columns per CTA).
//   warps 2-5   softmax: thread r owns query row r (= TMEM lane r), so the
//               row max / sum need no cross-thread reduction. It loads S_j,
//               masks (key in the sequence, |i − j| <= window/2 for sliding
//               layers), writes P_j = exp2(S·scale·log2e − m) as 16-bit values
//               packed two per column over the first 32 columns of S_j's
//               buffer, and — only when the running max grew by more than
//               2^8 — rescales O in TMEM once P_{j−1}·V_{j−1} is done. An
//               item's O is normalised by the row sum and stored to [T, H]
//               after the next item's first block has been handed over (its
//               last P·V completes meanwhile); the P·V that next overwrites
//               that O buffer (two items later) waits for that through the
//               P-ready barrier.
// Every barrier counts phases with per-role counters that run across work
// items; every mbarrier wait is bounded (2 s); a timeout sets g_attn_err and
// all roles unwind.
//
// MODE 0 / 1: the fused encoder's varlen attention (global / sliding window)
// over the [T, 3H] projection. MODE 2: the contract's sdpa
// (packages/tensor-backend/src/index.ts:230-237) on padded [B, nh, L, 64]
// q / k / v views of any 16-byte strides, read through 4-D tensor maps, with
// the bool mask (broadcast to [B, nh, Lq, Lk]) packed by a pre-pass
// (k_mask_pack) into one bit per key — rows [B][mask heads][mask rows][Lk/32]
// words, 8x fewer bytes than the mask — together with each (batch, mask head,
// query tile)'s range of key blocks holding a visible key; only those blocks
// are visited, and each softmax thread loads its row's two words of the next
// block while it works on the current one; the
// output is written as [B, Lq, nh, 64] rows, which the caller returns as the
// transposed [B, nh, Lq, 64] view (ModernBert.layer's transpose + reshape
// back to [B, L, H] then moves no bytes).
#include "lc_api.h"
#include "lc_gemm.h"
#include "lc_sm100.cuh"

#include <algorithm>
#include <cstdlib>

__device__ unsigned int g_attn_err;

using namespace sm100;

namespace {

constexpr int TQ = 128, TK = 64, HD = 64;
constexpr uint32_t TILE_BYTES = TQ * HD * 2;  // the 128 x 64 Q tile
constexpr uint32_t KV_BYTES = TK * HD * 2;    // one 64 x 64 K or V tile
constexpr uint32_t TMEM_COLS = 256;           // S double buffer (2 x 64) + O double buffer (2 x 64): two CTAs fit an SM
constexpr int NS = 2;                         // S buffers
constexpr uint32_t O_COL = NS * TK;           // O of work item t at O_COL + (t & 1) * HD
constexpr int NST = 4;                        // K/V ring depth
constexpr size_t ATTN_SMEM = 2 * TILE_BYTES + 2 * NST * KV_BYTES + 1024 + 256;
#ifndef LC_EXP_FMA_MASK
#define LC_EXP_FMA_MASK 0x8888u
#endif
// pairs i (of 16 per 32-key chunk) whose exponentials run on the FMA pipe
constexpr uint32_t kExpFmaMask = LC_EXP_FMA_MASK;

struct AttnTcArgs {
  const int4* tiles;  // (first token of the sequence, its length, first query row (multiple of 128), 0)
  void* out;          // [T, H] (MODE 2: [B, Lq, nh, 64])
  int H;
  int half_window;  // < 0: global attention
  float scale_log2;
  int heads;
  int nwork;  // tiles x heads (MODE 2: B x heads x query tiles)
  // MODE 2 only
  int Lq, Lk, nqt, mheads;
  const uint32_t* mbits;  // visible-key bits [B][mheads][mrows][mwords] (bit i of word w = key 32w + i); null = every key visible
  int mrows, mwords;      // mask rows: Lq, or 1 when the mask is the same for every query
  const int2* ranges;     // per (b, mask head, query tile, or one per (b, mask head) when mrows == 1): first key block,
                          // block count (null: every block)
};

struct Work {
  int tok0, L, q0, h, kv_lo, nb, b;
};

template <int MODE>
__device__ __forceinline__ Work decode(const AttnTcArgs& a, int4 t, int w) {
  Work r;
  if constexpr (MODE == 2) {
    r.h = w % a.heads;
    const int rest = w / a.heads, qt = rest % a.nqt;
    r.b = rest / a.nqt;
    r.tok0 = 0;
    r.L = a.Lq;
    r.q0 = qt * TQ;
    const int64_t bm = (int64_t)r.b * a.mheads + (a.mheads > 1 ? r.h : 0);
    const int2 rg = a.ranges ? a.ranges[a.mrows > 1 ? bm * a.nqt + qt : bm] : make_int2(0, (a.Lk + TK - 1) / TK);
    r.kv_lo = rg.x * TK;
    r.nb = max(rg.y, 1);  // a tile with no visible key still runs one (fully masked) block
    return r;
  }
  r.b = 0;
  r.tok0 = t.x;
  r.L = t.y;
  r.q0 = t.z;
  r.h = w % a.heads;
  int lo = 0, hi = r.L;
  if (MODE == 1) {
    lo = max(0, r.q0 - a.half_window);
    hi = min(r.L, r.q0 + TQ + a.half_window);
  }
  r.kv_lo = (lo / TK) * TK;
  r.nb = (hi - r.kv_lo + TK - 1) / TK;  // >= 1: q0 < L
  return r;
}

// One role's walk over this CTA's work items (w = blockIdx.x + t * gridDim.x);
// the tile entry of the following item is loaded one item ahead.
template <int MODE>
struct Items {
  int w, t;
  Work cur;
  int4 next;
  __device__ __forceinline__ int4 tile_of(const AttnTcArgs& a, int wi) const {
    if constexpr (MODE == 2) return make_int4(0, 0, 0, 0);
    return a.tiles[wi / a.heads];
  }
  __device__ __forceinline__ void start(const AttnTcArgs& a) {
    w = blockIdx.x;
    t = 0;
    if (w < a.nwork) cur = decode<MODE>(a, tile_of(a, w), w);
    const int wn = w + (int)gridDim.x;
    if (wn < a.nwork) next = tile_of(a, wn);
  }
  __device__ __forceinline__ bool valid(const AttnTcArgs& a) const { return w < a.nwork; }
  __device__ __forceinline__ void step(const AttnTcArgs& a) {
    w += gridDim.x;
    t++;
    if (w < a.nwork) cur = decode<MODE>(a, next, w);
    const int wn = w + (int)gridDim.x;
    if (wn < a.nwork) next = tile_of(a, wn);
  }
};

// Bit i set when byte i of w is nonzero (i < 4).
__device__ __forceinline__ uint32_t nonzero_bits4(uint32_t w) { return ((__vcmpne4(w, 0u) & 0x01010101u) * 0x10204080u) >> 28; }

// MODE 2: the two visibility words of query row qi (batch b, head h) for the
// key block starting at kbase (bit i of word c = key kbase + 32c + i).
__device__ __forceinline__ uint2 mask_words(const AttnTcArgs& a, int b, int h, int qi, int kbase) {
  if (qi >= a.Lq) return make_uint2(0u, 0u);
  if (!a.mbits) {
    const int n = min(TK, a.Lk - kbase);
    return make_uint2(n >= 32 ? 0xffffffffu : (0xffffffffu >> (32 - n)), n >= 64 ? 0xffffffffu : (n > 32 ? (0xffffffffu >> (64 - n)) : 0u));
  }
  const uint32_t* row = a.mbits + (((int64_t)b * a.mheads + (a.mheads > 1 ? h : 0)) * a.mrows + (a.mrows > 1 ? qi : 0)) * a.mwords;
  const int w = kbase >> 5;
  return make_uint2(__ldg(row + w), w + 1 < a.mwords ? __ldg(row + w + 1) : 0u);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 2^x for a pair on the FMA and integer pipes (the exponential unit does one
// value per lane every 8 cycles per SM sub-partition, the FMA pipe 32 per
// cycle): x = n + f with n = round(x) (the 1.5·2^23 shift), f in [-1/2, 1/2];
// 2^f by a cubic fitted here for relative error (|error| < 7.8e-5, below the
// half-ulp 2^-11 of the f16 P it feeds); 2^n added to the exponent bits.
// x is clamped to >= -126 (2^-126 rounds to 0 in the 16-bit P).
__device__ __forceinline__ float2 exp2_fma2(float2 x) {
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const float2 M = make_float2(12582912.f, 12582912.f);  // 1.5 * 2^23
  const float2 t = add2(x, M);
  const float2 n = add2(t, make_float2(-12582912.f, -12582912.f));
  const float2 f = add2(x, make_float2(-n.x, -n.y));
  float2 p = fma2(make_float2(0.05508868f, 0.05508868f), f, make_float2(0.24260405f, 0.24260405f));
  p = fma2(p, f, make_float2(0.6932762f, 0.6932762f));
  p = fma2(p, f, make_float2(0.99992895f, 0.99992895f));
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (std::is_same<T, __half>::value) {
    __half2 h = __floats2half2_rn(a, b);
    return *(uint32_t*)&h;
  } else {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *(uint32_t*)&h;
  }
}

template <typename T, int MODE>
__global__ void __launch_bounds__(192, 2) k_attn_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                                                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ AttnTcArgs a) {
  constexpr bool LOCAL = MODE == 1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = smem;                 // 2 buffers
  uint8_t* sK = sQ + 2 * TILE_BYTES;  // NST stages
  uint8_t* sV = sK + NST * KV_BYTES;  // NST stages
  uint64_t* bars = (uint64_t*)(sV + NST * KV_BYTES);
  uint64_t* q_full = bars;            // [2]
  uint64_t* q_empty = q_full + 2;     // [2]
  uint64_t* kv_full = q_empty + 2;    // [NST]
  uint64_t* kv_empty = kv_full + NST; // [NST]
  uint64_t* s_full = kv_empty + NST;  // [NS]
  uint64_t* p_ready = s_full + NS;    // [NS]
  // P_g·V_g commits to o_done[g & 1]: a softmax warp waiting for block g is
  // never more than one phase behind (P_{g+2}·V_{g+2} needs P_{g+2}, which
  // that warp has not produced yet).
  uint64_t* o_done = p_ready + NS;  // [2]
  uint32_t* tmem_slot = (uint32_t*)(o_done + 2);
  volatile int* abort = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; i++) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&o_done[i], 1);
    }
    for (int i = 0; i < NS; i++) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 4);
    }
    for (int i = 0; i < NST; i++) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmQ) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmKV) : "memory");
    if (MODE == 2) asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmV) : "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // the projection that wrote q, k, v has completed

  if (warp == 0) {
    if (lane == 0) {
      int issued[NST], q_issued[2] = {0, 0};
      uint32_t iph[NST], q_ph[2] = {0, 0};
      for (int s = 0; s < NST; s++) issued[s] = 0, iph[s] = 0;
      uint32_t kv_it = 0;
      bool ok = true;
      Items<MODE> it;
      for (it.start(a); ok && it.valid(a); it.step(a)) {
        const Work& wk = it.cur;
        const int t = it.t, qb = t & 1;
        if (!mbar_wait(&q_empty[qb], ((t >> 1) & 1) ^ 1, abort, &g_attn_err)) break;
        mbar_arrive_expect_tx(&q_full[qb], TILE_BYTES);
        if constexpr (MODE == 2) tma_load_4d(sQ + qb * TILE_BYTES, &tmQ, &q_full[qb], 0, wk.q0, wk.h, wk.b);
        else tma_load_2d(sQ + qb * TILE_BYTES, &tmQ, &q_full[qb], wk.h * HD, wk.tok0 + wk.q0);
        q_issued[qb] = 1;
        q_ph[qb] = (t >> 1) & 1;
        for (int j = 0; j < wk.nb; j++, kv_it++) {
          const int st = kv_it % NST;
          const uint32_t ph = (kv_it / NST) & 1;
          if (!mbar_wait(&kv_empty[st], ph ^ 1, abort, &g_attn_err)) { ok = false; break; }
          mbar_arrive_expect_tx(&kv_full[st], 2 * KV_BYTES);
          const int row = wk.tok0 + wk.kv_lo + j * TK;
          if constexpr (MODE == 2) {
            tma_load_4d(sK + st * KV_BYTES, &tmKV, &kv_full[st], 0, row, wk.h, wk.b);
            tma_load_4d(sV + st * KV_BYTES, &tmV, &kv_full[st], 0, row, wk.h, wk.b);
          } else {
            tma_load_2d(sK + st * KV_BYTES, &tmKV, &kv_full[st], a.H + wk.h * HD, row);
            tma_load_2d(sV + st * KV_BYTES, &tmKV, &kv_full[st], 2 * a.H + wk.h * HD, row);
          }
          issued[st] = 1;
          iph[st] = ph;
        }
      }
      // drain: every copy issued here has landed before the CTA can exit
      for (int qb = 0; qb < 2; qb++)
        if (q_issued[qb]) {
          const uint64_t t0 = gtimer();
          while (!mbar_try_wait(&q_full[qb], q_ph[qb]) && gtimer() - t0 < kWaitNs) {}
        }
      for (int s = 0; s < NST; s++)
        if (issued[s]) {
          const uint64_t t0 = gtimer();
          while (!mbar_try_wait(&kv_full[s], iph[s]) && gtimer() - t0 < kWaitNs) {}
        }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // Issue order over the CTA's stream of key blocks g = 0, 1, ... (across
      // work items):  S_0 .. S_{NS-1}, then for each g: [P_g ready] P_g·V_g,
      // S_{g+NS}. S_{g+NS} reuses the buffer of S_g, whose P the P_g·V_g
      // issued just before reads first (tcgen05 MMAs of one thread run in
      // issue order); the softmax has finished with S_g (P_g ready).
      const uint32_t id_s = idesc_f16<T, TK>();
      const uint32_t id_pv = idesc_f16<T, HD, 128, true>();
      const uint64_t dq0 = sdesc_sw128(smem_u32(sQ)), dk0 = sdesc_sw128(smem_u32(sK)), dv0 = sdesc_sw128_mn(smem_u32(sV));
      uint64_t* last_bar = nullptr;  // the barrier of the most recent commit, for the drain
      uint32_t last_ph = 0;
      Items<MODE> si, pi;  // S cursor and P·V cursor
      si.start(a);
      pi.start(a);
      int sj = 0, pj = 0;
      uint32_t sg = 0, pg = 0;
      auto issue_s = [&]() -> bool {
        const int qb = si.t & 1;
        if (sj == 0) {
          if (!mbar_wait(&q_full[qb], (si.t >> 1) & 1, abort, &g_attn_err)) return false;
        }
        const int st = sg % NST;
        if (!mbar_wait(&kv_full[st], (sg / NST) & 1, abort, &g_attn_err)) return false;
        tc_fence_after();
        const uint32_t d = tmem + (sg % NS) * TK;
        const uint64_t dq = dq0 + ((qb * TILE_BYTES) >> 4), dk = dk0 + ((st * KV_BYTES) >> 4);
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) tc_mma(d, dq + kk * 2, dk + kk * 2, id_s, kk > 0 ? 1u : 0u);
        tc_commit(&s_full[sg % NS]);
        last_bar = &s_full[sg % NS];
        last_ph = (sg / NS) & 1;
        if (sj == si.cur.nb - 1) tc_commit(&q_empty[qb]);
        sg++;
        if (++sj == si.cur.nb) {
          sj = 0;
          si.step(a);
        }
        return true;
      };
      bool ok = true;
      for (int i = 0; i < NS && ok && si.valid(a); i++) ok = issue_s();
      while (ok && pi.valid(a)) {
        const uint32_t b = pg % NS;
        if (!mbar_wait(&p_ready[b], (pg / NS) & 1, abort, &g_attn_err)) break;
        tc_fence_after();
        const int st = pg % NST;
        const uint64_t dv = dv0 + ((st * KV_BYTES) >> 4);
#pragma unroll
        for (int kk = 0; kk < TK / 16; kk++)
          tc_mma_ts(tmem + O_COL + (pi.t & 1) * HD, tmem + b * TK + kk * 8, dv + kk * (2048 >> 4), id_pv, (pj > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&o_done[pg & 1]);
        tc_commit(&kv_empty[st]);
        last_bar = &o_done[pg & 1];
        last_ph = (pg >> 1) & 1;
        pg++;
        if (++pj == pi.cur.nb) {
          pj = 0;
          pi.step(a);
        }
        if (si.valid(a)) ok = issue_s();
      }
      if (last_bar) {  // MMAs complete in issue order: the last commit covers them all
        const uint64_t t0 = gtimer();
        while (!mbar_try_wait(last_bar, last_ph) && gtimer() - t0 < kWaitNs) {}
      }
    }
  } else {
    // softmax / correction / epilogue: thread <-> query row
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl = a.scale_log2;
    uint32_t g = 0;
    bool ok = true;
    // O is double-buffered by work-item parity: a finished item's rows are
    // normalised and stored after the first block of the next item has been
    // handed to the MMA warp, so the softmax does not idle while the item's
    // last P·V completes. The next P·V into that buffer (two items later)
    // waits for a P-ready arrival that follows this store.
    bool pend = false;
    uint32_t pend_gl = 0, pend_ocol = 0;
    float pend_inv = 0.f;
    T* pend_out = nullptr;  // null: this row is past its sequence end
    auto flush = [&]() -> bool {
      if (!mbar_wait(&o_done[pend_gl & 1], (pend_gl >> 1) & 1, abort, &g_attn_err)) return false;
      tc_fence_after();
      uint32_t r[HD];
      tmem_ld64(tmem + lane_off + pend_ocol, r);
      tmem_wait_ld();
      if (pend_out) {
#pragma unroll
        for (int q = 0; q < HD / 8; q++) {
          uint4 v;
          uint32_t* pv = (uint32_t*)&v;
#pragma unroll
          for (int i = 0; i < 4; i++)
            pv[i] = pack2<T>(__uint_as_float(r[q * 8 + 2 * i]) * pend_inv, __uint_as_float(r[q * 8 + 2 * i + 1]) * pend_inv);
          *(uint4*)(pend_out + q * 8) = v;
        }
      }
      pend = false;
      return true;
    };
    Items<MODE> it;
    for (it.start(a); ok && it.valid(a); it.step(a)) {
      const Work& wk = it.cur;
      const int qi = wk.q0 + row;
      const uint32_t ocol = O_COL + (it.t & 1) * HD;
      const bool warp_live = wk.q0 + quarter * 32 < wk.L;  // warps wholly past the sequence end skip their exps
      float m = -INFINITY, l = 0.f;
      uint2 mw_next = make_uint2(0u, 0u);  // MODE 2: this row's visibility words of the next block
      if constexpr (MODE == 2) mw_next = mask_words(a, wk.b, wk.h, qi, wk.kv_lo);
      for (int j = 0; j < wk.nb; j++) {
        const uint32_t gj = g + j, b = gj % NS;
        if (!mbar_wait(&s_full[b], (gj / NS) & 1, abort, &g_attn_err)) { ok = false; break; }
        tc_fence_after();
        const int kbase = wk.kv_lo + j * TK;
        // this row's visible keys, relative to the block: [lo, hi]
        const int lo = (LOCAL ? max(0, qi - a.half_window) : 0) - kbase;
        const int hi = (LOCAL ? min(wk.L - 1, qi + a.half_window) : wk.L - 1) - kbase;
        // per 32-key chunk, warp-uniform: live = some row sees a key of it; full = every row sees all of it
        bool live[TK / 32], full[TK / 32];
        // per chunk, this row's visible keys as a bit mask (bit i = key c·32 + i of the block)
        uint32_t vis[TK / 32];
        if constexpr (MODE == 2) {
          vis[0] = mw_next.x;
          vis[1] = mw_next.y;
          if (j + 1 < wk.nb) mw_next = mask_words(a, wk.b, wk.h, qi, kbase + TK);  // in flight during this block
#pragma unroll
          for (int c = 0; c < TK / 32; c++) {
            live[c] = warp_live && __any_sync(0xffffffffu, vis[c] != 0u);
            full[c] = __all_sync(0xffffffffu, vis[c] == 0xffffffffu);
          }
        } else {
#pragma unroll
          for (int c = 0; c < TK / 32; c++) {
            const int c0 = c * 32, c1 = c0 + 31;
            if (LOCAL) {
              live[c] = warp_live && __any_sync(0xffffffffu, c1 >= lo && c0 <= hi);
              full[c] = __all_sync(0xffffffffu, c0 >= lo && c1 <= hi);
            } else {  // every row sees keys [0, L): lo <= 0 and hi are the same for the whole warp
              live[c] = warp_live && c0 <= hi;
              full[c] = c1 <= hi;
            }
          }
#pragma unroll
          for (int c = 0; c < TK / 32; c++) {
            const int a0 = max(lo - c * 32, 0), a1 = min(hi - c * 32, 31);
            vis[c] = a0 <= a1 ? ((0xffffffffu >> (31 - a1)) & (0xffffffffu << a0)) : 0u;
          }
        }
        float s[TK];
        {
          uint32_t sr[TK];
          tmem_ld64(tmem + lane_off + b * TK, sr);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < TK; i++) s[i] = __uint_as_float(sr[i]);
        }
        // row max of the raw scores (the softmax scale is positive, so it
        // commutes), four independent chains of three-input maxima
        float mc[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < TK / 32; c++) {
          if (!live[c]) continue;
          if (full[c]) {
#pragma unroll
            for (int i = 0; i < 16; i++) mc[i & 3] = max3(mc[i & 3], s[c * 32 + 2 * i], s[c * 32 + 2 * i + 1]);
          } else {
#pragma unroll
            for (int i = 0; i < 16; i++) {
              const int k = c * 32 + 2 * i;
              const float v0 = (vis[c] >> (2 * i)) & 1u ? s[k] : -INFINITY;
              const float v1 = (vis[c] >> (2 * i + 1)) & 1u ? s[k + 1] : -INFINITY;
              mc[i & 3] = max3(mc[i & 3], v0, v1);
            }
          }
        }
        const float mx = max3(mc[0], mc[1], fmaxf(mc[2], mc[3]));
        // lazy rescale: the reference max (raw units) only moves when it grew by more
        // than 2^8 after scaling, so P stays below 256 and O needs rescaling rarely
        const float m_new = fmaxf(m, mx);
        const bool grow = (m_new - m) * sl > 8.f;  // m = -inf: true unless the row is still all masked
        const float corr = grow ? ex2((m - m_new) * sl) : 1.f;
        if (grow) m = m_new;
        const float nbias = m == -INFINITY ? 0.f : -m * sl;
        float2 acc[4] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
        uint32_t pr[TK / 2];  // P as 16-bit pairs, packed as the exponentials are computed
#pragma unroll
        for (int c = 0; c < TK / 32; c++) {
          if (live[c] && full[c]) {
#pragma unroll
            for (int i = 0; i < 16; i++) {
              const int k = c * 32 + 2 * i;
              float2 x = fma2(make_float2(s[k], s[k + 1]), make_float2(sl, sl), make_float2(nbias, nbias));
              if (kExpFmaMask & (1u << i)) {  // part of the pairs on the FMA pipe
                x = exp2_fma2(x);
              } else {
                x.x = ex2(x.x);
                x.y = ex2(x.y);
              }
              pr[c * 16 + i] = pack2<T>(x.x, x.y);
              acc[i & 3] = add2(acc[i & 3], x);
            }
          } else if (live[c]) {
#pragma unroll
            for (int i = 0; i < 16; i++) {
              const int k = c * 32 + 2 * i;
              float2 x = fma2(make_float2(s[k], s[k + 1]), make_float2(sl, sl), make_float2(nbias, nbias));
              x.x = ex2(x.x);
              x.y = ex2(x.y);
              x.x = (vis[c] >> (2 * i)) & 1u ? x.x : 0.f;  // keys outside the row's range contribute 0
              x.y = (vis[c] >> (2 * i + 1)) & 1u ? x.y : 0.f;
              pr[c * 16 + i] = pack2<T>(x.x, x.y);
              acc[i & 3] = add2(acc[i & 3], x);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 16; i++) pr[c * 16 + i] = 0u;
          }
        }
        const float2 a01 = add2(acc[0], acc[1]), a23 = add2(acc[2], acc[3]);
        const float2 at = add2(a01, a23);
        l = fmaf(l, corr, at.x + at.y);
        tmem_st32(tmem + lane_off + b * TK, pr);
        tmem_wait_st();
        if (j >= 1 && __any_sync(0xffffffffu, grow)) {
          // O holds blocks < j once P_{j-1}·V_{j-1} is done; rescale it before P_j·V_j
          const uint32_t gp = gj - 1;
          if (!mbar_wait(&o_done[gp & 1], (gp >> 1) & 1, abort, &g_attn_err)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < HD / 32; c++) {
            uint32_t r[32];
            tmem_ld32(tmem + lane_off + ocol + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; i++) r[i] = __float_as_uint(__uint_as_float(r[i]) * corr);
            tmem_st32(tmem + lane_off + ocol + c * 32, r);
          }
          tmem_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_ready[b]);
        if (j == 0 && pend && !flush()) { ok = false; break; }
      }
      if (!ok) break;
      pend = true;
      pend_gl = g + wk.nb - 1;
      pend_ocol = ocol;
      pend_inv = l > 0.f ? 1.f / l : 0.f;  // a row with no visible key (undefined by the contract) gives zeros
      if constexpr (MODE == 2)
        pend_out = qi < wk.L ? (T*)a.out + (((int64_t)wk.b * a.Lq + qi) * a.heads + wk.h) * HD : nullptr;
      else
        pend_out = qi < wk.L ? (T*)a.out + ((int64_t)wk.tok0 + qi) * a.H + wk.h * HD : nullptr;
      g += wk.nb;
    }
    if (ok && pend) flush();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

template <typename T, int MODE>
void launch_attn(const CUtensorMap& mq, const CUtensorMap& mkv, const CUtensorMap& mv, const AttnTcArgs& a, cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    CUDA_OK(cudaFuncSetAttribute(k_attn_tc<T, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ATTN_SMEM));
    attr = true;
  }
  const int grid = std::min(a.nwork, 2 * lc::num_sms());  // persistent: two CTAs per SM
  lc::launch_chain(k_attn_tc<T, MODE>, dim3((unsigned)grid), dim3(192), ATTN_SMEM, st, mq, mkv, mv, a);
}

// MODE 2 pre-pass: packs the bool mask (element strides s0..s3 over
// [B, nh, Lq, Lk], 0 where broadcast) into visibility bits [B][mheads][mrows][mwords]
// and records, for each 128-row group of mask rows (a query tile, or the one
// row when mrows == 1), the first key block holding a key visible to some row
// of the group and the number of blocks up to the last such block (0: none).
// One 128-thread block per (b, mask head, row group), thread = mask row.
__global__ void __launch_bounds__(TQ) k_mask_pack(const uint8_t* mask, long long s0, long long s1, long long s2, long long s3, int mheads,
                                                  int mrows, int Lk, int mwords, uint32_t* bits, int2* ranges) {
  pdl_trigger();
  pdl_wait();
  const int ngroups = (mrows + TQ - 1) / TQ;
  const int gi = blockIdx.x % ngroups, bm = blockIdx.x / ngroups, mh = bm % mheads, b = bm / mheads;
  const int r = gi * TQ + (int)threadIdx.x;
  int first = INT_MAX, last = -1;
  if (r < mrows) {
    const uint8_t* row = mask + (int64_t)b * s0 + (int64_t)mh * s1 + (int64_t)r * s2;
    uint32_t* out = bits + ((int64_t)bm * mrows + r) * mwords;
    const bool vec = s3 == 1 && (((uintptr_t)row) & 15) == 0;
    for (int w = 0; w < mwords; w++) {
      const int k0 = w * 32;
      uint32_t v = 0;
      if (vec && k0 + 32 <= Lk) {
        const uint4 u0 = __ldg((const uint4*)(row + k0)), u1 = __ldg((const uint4*)(row + k0) + 1);
        v = nonzero_bits4(u0.x) | (nonzero_bits4(u0.y) << 4) | (nonzero_bits4(u0.z) << 8) | (nonzero_bits4(u0.w) << 12) |
            (nonzero_bits4(u1.x) << 16) | (nonzero_bits4(u1.y) << 20) | (nonzero_bits4(u1.z) << 24) | (nonzero_bits4(u1.w) << 28);
      } else {
        for (int i = 0; i < 32 && k0 + i < Lk; i++)
          if (row[(int64_t)(k0 + i) * s3]) v |= 1u << i;
      }
      out[w] = v;
      if (v) {
        if (first == INT_MAX) first = k0 + __ffs(v) - 1;
        last = k0 + 31 - __clz(v);
      }
    }
  }
  __shared__ int lo_s, hi_s;
  if (threadIdx.x == 0) lo_s = INT_MAX, hi_s = -1;
  __syncthreads();
  if (first != INT_MAX) atomicMin(&lo_s, first);
  if (last >= 0) atomicMax(&hi_s, last);
  __syncthreads();
  if (threadIdx.x == 0) {
    if (hi_s < 0) ranges[blockIdx.x] = make_int2(0, 0);
    else ranges[blockIdx.x] = make_int2(lo_s / TK, hi_s / TK - lo_s / TK + 1);
  }
}

}  // namespace

namespace lc {

// Work list of the tcgen05 kernel: one entry per 128-row query tile, longest
// sequences first (the persistent CTAs take items in this order, so the
// costly ones start early and the short ones fill the tail).
std::vector<int4> attention_tiles_tc(const int32_t* cu, int nseq) {
  std::vector<int4> t;
  for (int s = 0; s < nseq; s++) {
    int L = cu[s + 1] - cu[s];
    for (int q0 = 0; q0 < L; q0 += TQ) t.push_back(make_int4(cu[s], L, q0, 0));
  }
  std::stable_sort(t.begin(), t.end(), [](const int4& x, const int4& y) { return x.y > y.y; });
  return t;
}

void attention_varlen_tc(const void* qkv, void* out, const int4* tiles_dev, int ntiles, int64_t T, int H, int half_window, float scale,
                         int dtype, cudaStream_t st) {
  LC_CHECK(H % HD == 0 && T < INT32_MAX, "attention: head dim must be 64");
  if (ntiles == 0) return;
  LC_CHECK(ntiles < (1 << 30), "attention: too many tiles");
  const CUtensorMap& mq = tensor_map_2d(qkv, T, 3 * (int64_t)H, 3 * (int64_t)H, 64, TQ, dtype);
  const CUtensorMap& mkv = tensor_map_2d(qkv, T, 3 * (int64_t)H, 3 * (int64_t)H, 64, TK, dtype);
  const int heads = H / HD;
  LC_CHECK((int64_t)ntiles * heads < INT32_MAX, "attention: too many work items");
  AttnTcArgs a{};
  a.tiles = tiles_dev;
  a.out = out;
  a.H = H;
  a.half_window = half_window;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.heads = heads;
  a.nwork = ntiles * heads;
  if (dtype == LC_F16) {
    if (half_window >= 0) launch_attn<__half, 1>(mq, mkv, mkv, a, st);
    else launch_attn<__half, 0>(mq, mkv, mkv, a, st);
  } else {
    if (half_window >= 0) launch_attn<__nv_bfloat16, 1>(mq, mkv, mkv, a, st);
    else launch_attn<__nv_bfloat16, 0>(mq, mkv, mkv, a, st);
  }
  LC_LAUNCHED(1);
}

namespace {
// 4-D map over a [B, nh, L, 64] view (element strides s[0..2] for B, nh, L;
// innermost stride 1): dims (64, L, nh, B), box 64 x rows x 1 x 1, 128-byte swizzle.
bool map_bhld(CUtensorMap* m, const void* ptr, int dtype, int64_t B, int64_t nh, int64_t L, const int64_t* s0, int rows) {
  // a dimension of extent 1 is never stepped: its stride (which a view may
  // carry as 0 or anything) is replaced by 16 bytes for the map
  const int64_t ext[3] = {B, nh, L};
  int64_t s[3];
  for (int i = 0; i < 3; i++) s[i] = ext[i] == 1 ? 8 : s0[i];
  for (int i = 0; i < 3; i++)
    if ((s[i] * 2) % 16 || s[i] <= 0 || s[i] * 2 >= ((int64_t)1 << 40)) return false;
  if (((uintptr_t)ptr) & 15) return false;
  cuuint64_t dims[4] = {64, (cuuint64_t)L, (cuuint64_t)nh, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(s[2] * 2), (cuuint64_t)(s[1] * 2), (cuuint64_t)(s[0] * 2)};
  cuuint32_t box[4] = {64, (cuuint32_t)rows, 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = tensor_map_encoder()(m, dtype == LC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                                    const_cast<void*>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}
}  // namespace

// Packed masks are kept per mask view: a model passes the same mask tensor to
// every layer of a forward (ModernBert.encode hands each layer kind's mask to
// all its layers), so the bits and key-block ranges are built once. The key is
// the storage (unique id and write version) and the broadcast view; an entry
// goes when its storage is released. Entries made while a CUDA graph is being
// captured live only inside that capture (their buffers are the graph's own
// allocations, freed inside it at the end) and entries made outside it are
// not used by it, so a recording never holds a pointer the cache may free.
namespace {
struct PackedMask {
  uint64_t sid;
  uint32_t ver;
  const void* ptr;
  int64_t strides[4];
  int64_t dims[4];
  int mheads, mrows, mwords;
  uint32_t* bits;
  int2* ranges;
  bool in_capture;
};
std::vector<PackedMask>& mask_cache() {
  static std::vector<PackedMask> v;
  return v;
}
constexpr size_t kMaskCacheEntries = 8;
void drop_mask(size_t i, bool free_buffers) {
  auto& c = mask_cache();
  if (free_buffers) {
    dfree(c[i].bits);
    dfree(c[i].ranges);
  }
  c.erase(c.begin() + (std::ptrdiff_t)i);
}
}  // namespace

void storage_released(uint64_t id) {
  auto& c = mask_cache();
  for (size_t i = c.size(); i-- > 0;)
    if (c[i].sid == id) drop_mask(i, true);
}
void capture_ending(bool aborted) {
  auto& c = mask_cache();
  for (size_t i = c.size(); i-- > 0;)
    if (c[i].in_capture) drop_mask(i, !aborted);
}

// LAYA_CUDA_SDPA_TC=0 keeps the contract's sdpa on the mma.sync kernel.
static bool sdpa_tc_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("LAYA_CUDA_SDPA_TC");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

bool sdpa_tc(const LcTensor* q, const LcTensor* k, const LcTensor* v, const LcTensor* m, float scale, LcTensor** out) {
  if (!sdpa_tc_enabled()) return false;
  if (!is_half(q->dtype) || k->dtype != q->dtype || v->dtype != q->dtype) return false;
  const int64_t B = q->shape[0], nh = q->shape[1], Lq = q->shape[2], Lk = k->shape[2];
  if (q->shape[3] != HD || k->shape[3] != HD || v->shape[3] != HD || Lq < 1 || Lk < 1) return false;
  if (Lq > INT32_MAX / 2 || Lk > INT32_MAX / 2 || B * nh > INT32_MAX || nh > INT32_MAX) return false;
  for (const LcTensor* t : {q, k, v})
    if (t->strides[3] != 1) return false;
  CUtensorMap mq, mk, mv;
  if (!map_bhld(&mq, q->data(), q->dtype, B, nh, Lq, q->strides, TQ) || !map_bhld(&mk, k->data(), k->dtype, B, nh, Lk, k->strides, TK) ||
      !map_bhld(&mv, v->data(), v->dtype, B, nh, Lk, v->strides, TK))
    return false;
  const int64_t nqt = (Lq + TQ - 1) / TQ;
  if (B * nh * nqt >= INT32_MAX) return false;
  AttnTcArgs a{};
  a.heads = (int)nh;
  a.H = (int)(nh * HD);
  a.half_window = -1;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.Lq = (int)Lq;
  a.Lk = (int)Lk;
  a.nqt = (int)nqt;
  a.nwork = (int)(B * nh * nqt);
  cudaStream_t st = stream();
  // visibility bits and key-block ranges per (batch, mask head, query tile);
  // without a mask every key of every block is visible
  uint32_t* mbits = nullptr;
  int2* ranges = nullptr;
  bool cached = false;
  a.mheads = 1;
  a.mrows = 1;
  if (m) {
    TV mtv = tv_broadcast(m, {B, nh, Lq, Lk});
    const int mheads = mtv.strides[1] == 0 ? 1 : (int)nh;
    const int mrows = mtv.strides[2] == 0 ? 1 : (int)Lq;
    const int mwords = (int)((Lk + 31) / 32);
    const int64_t ngroups = (mrows + TQ - 1) / TQ;
    const int64_t nblocks = B * mheads * ngroups;
    if (nblocks >= INT32_MAX) return false;
    const bool capturing = lc::capturing();
    const bool cacheable = !m->st->external && m->st->id != 0;
    const int64_t dims[4] = {B, nh, Lq, Lk};
    auto& c = mask_cache();
    for (const PackedMask& e : c)
      if (cacheable && e.sid == m->st->id && e.ver == m->st->version && e.ptr == mtv.ptr && e.in_capture == capturing &&
          std::equal(e.strides, e.strides + 4, mtv.strides) && std::equal(e.dims, e.dims + 4, dims)) {
        mbits = e.bits;
        ranges = e.ranges;
        cached = true;
        break;
      }
    if (!cached) {
      mbits = (uint32_t*)dmalloc((size_t)B * mheads * mrows * mwords * sizeof(uint32_t));
      ranges = (int2*)dmalloc((size_t)nblocks * sizeof(int2));
      lc::launch_chain(k_mask_pack, dim3((unsigned)nblocks), dim3(TQ), 0, st, (const uint8_t*)mtv.ptr, mtv.strides[0], mtv.strides[1],
                       mtv.strides[2], mtv.strides[3], mheads, mrows, (int)Lk, mwords, mbits, ranges);
      LC_LAUNCHED(1);
      if (cacheable) {
        if (!capturing && c.size() >= kMaskCacheEntries)
          for (size_t i = 0; i < c.size(); i++)
            if (!c[i].in_capture) {
              drop_mask(i, true);
              break;
            }
        PackedMask e{m->st->id, m->st->version, mtv.ptr, {}, {}, mheads, mrows, mwords, mbits, ranges, capturing};
        std::copy(mtv.strides, mtv.strides + 4, e.strides);
        std::copy(dims, dims + 4, e.dims);
        c.push_back(e);
        cached = true;
      }
    }
    a.mheads = mheads;
    a.mrows = mrows;
    a.mwords = mwords;
  }
  a.mbits = mbits;
  a.ranges = ranges;
  // output rows [B, Lq, nh, 64], returned as the [B, nh, Lq, 64] view
  LcTensor* y = alloc(q->dtype, {B, Lq, nh, HD});
  a.out = y->data();
  if (q->dtype == LC_F16) launch_attn<__half, 2>(mq, mk, mv, a, st);
  else launch_attn<__nv_bfloat16, 2>(mq, mk, mv, a, st);
  LC_LAUNCHED(1);
  if (!cached) {
    if (ranges) dfree(ranges);
    if (mbits) dfree(mbits);
  }
  *out = view_of(y, {B, nh, Lq, HD}, {Lq * nh * HD, HD, nh * HD, 1}, 0);
  release(y);
  return true;
}

std::string take_attention_errors() {
  unsigned int e = 0, z = 0;
  CUDA_OK(cudaMemcpyFromSymbol(&e, g_attn_err, sizeof(e)));
  if (!e) return "";
  CUDA_OK(cudaMemcpyToSymbol(g_attn_err, &z, sizeof(z)));
  return "tcgen05 attention: a pipeline wait timed out (kernel aborted its tile)";
}

}  // namespace lc

// Sets this unit's bounded-wait limit (lc_debug_set_wait_limit).
void lc_internal_wait_limit_attention(unsigned long long ns) { CUDA_OK(cudaMemcpyToSymbol(sm100::g_wait_limit_ns, &ns, sizeof(ns))); }
