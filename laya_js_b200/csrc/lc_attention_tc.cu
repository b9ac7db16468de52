// Tensor-core (tcgen05 / TMEM) flash attention over unpadded varlen sequences,
// head dim 64 — the attention of ModernBert.layer
// (packages/modernbert/src/index.ts:348-352: sdpa with the masks of
// attentionMasks, index.ts:240-259) computed without masks or padding.
//
// One CTA = 128 query rows of one (sequence, head); key blocks of 64.
//   warp 0      TMA producer: Q once, K and V blocks into a 2-stage ring
//               (128 x 64 tiles of the fused [T, 3H] projection, 128-byte swizzle);
//   warp 1      TMEM owner and single-thread MMA issuer:
//                 S_j = Q·K_jᵀ  (M=128, N=64, K=64; A, B from shared memory)
//                 O  += P_j·V_j (M=128, N=64, K=64; A = P from TMEM, B = V
//                                from shared memory, MN-major)
//               S is double-buffered in TMEM (columns 0-63 / 64-127), so
//               S_{j+1} runs while the softmax works on S_j; O lives at
//               columns 128-191 (256 columns per CTA: two CTAs share an SM).
//   warps 2-5   softmax: thread r owns query row r (= TMEM lane r), so the
//               row max / sum need no cross-thread reduction. It loads S_j,
//               masks (key in the sequence, |i − j| <= window/2 for sliding
//               layers), writes P_j = exp2(S·scale·log2e − m) as f16 over the
//               first 64 columns of S_j's buffer, and — only when the running
//               max grew — rescales O in TMEM once P_{j−1}·V_{j−1} is done.
//               At the end it normalises O by the row sum and stores [T, H].
// Every mbarrier wait is bounded (2 s); a timeout sets g_attn_err and unwinds.
#include "lc_api.h"
#include "lc_gemm.h"
#include "lc_sm100.cuh"

__device__ unsigned int g_attn_err;

using namespace sm100;

namespace {

constexpr int TQ = 128, TK = 64, HD = 64;
constexpr uint32_t TILE_BYTES = TQ * HD * 2;  // the 128 x 64 Q tile
constexpr uint32_t KV_BYTES = TK * HD * 2;    // one 64 x 64 K or V tile
constexpr uint32_t TMEM_COLS = 256;           // S double buffer (2 x 64) + O (64): two CTAs fit an SM
constexpr int NST = 5;                        // K/V ring depth: covers the TMA latency of several blocks
constexpr size_t ATTN_SMEM = TILE_BYTES + 2 * NST * KV_BYTES + 1024 + 256;

struct AttnTcArgs {
  const int4* tiles;  // (first token of the sequence, its length, first query row (multiple of 128), 0)
  void* out;          // [T, H]
  int H;
  int half_window;  // < 0: global attention
  float scale_log2;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
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

template <typename T, bool LOCAL>
__global__ void __launch_bounds__(192, 2) k_attn_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                                                    const __grid_constant__ AttnTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + TILE_BYTES;      // NST stages
  uint8_t* sV = sK + NST * KV_BYTES;  // NST stages
  uint64_t* bars = (uint64_t*)(sV + NST * KV_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;          // [NST]
  uint64_t* kv_empty = kv_full + NST;    // [NST]
  uint64_t* s_full = kv_empty + NST;     // [2]
  uint64_t* p_ready = s_full + 2;        // [2]
  // P_j·V_j commits to o_done[j & 1]: with two barriers a waiter is never more
  // than one phase behind (S_j complete implies P_{j-2}·V_{j-2} complete).
  uint64_t* o_done = p_ready + 2;  // [2]
  uint32_t* tmem_slot = (uint32_t*)(o_done + 2);
  volatile int* abort = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int4 tile = a.tiles[blockIdx.x];
  const int tok0 = tile.x, L = tile.y, q0 = tile.z, h = blockIdx.y;
  int kv_lo = 0, kv_hi = L;
  if (LOCAL) {
    kv_lo = max(0, q0 - a.half_window);
    kv_hi = min(L, q0 + TQ + a.half_window);
  }
  kv_lo = (kv_lo / TK) * TK;
  const int nb = (kv_hi - kv_lo + TK - 1) / TK;  // >= 1: q0 < L

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NST; i++) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 4);
      mbar_init(&o_done[i], 1);
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
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t o_col = 2 * TK;

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmQ) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmKV) : "memory");
      mbar_arrive_expect_tx(q_full, TILE_BYTES);
      tma_load_2d(sQ, &tmQ, q_full, h * HD, tok0 + q0);
      int issued[NST];
      uint32_t iph[NST];
      for (int s = 0; s < NST; s++) issued[s] = 0, iph[s] = 0;
      for (int j = 0; j < nb; j++) {
        const int st = j % NST;
        const uint32_t ph = (j / NST) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1, abort, &g_attn_err)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * KV_BYTES);
        const int row = tok0 + kv_lo + j * TK;
        tma_load_2d(sK + st * KV_BYTES, &tmKV, &kv_full[st], a.H + h * HD, row);
        tma_load_2d(sV + st * KV_BYTES, &tmKV, &kv_full[st], 2 * a.H + h * HD, row);
        issued[st] = 1;
        iph[st] = ph;
      }
      // drain: every copy issued here has landed before the CTA can exit
      uint64_t t0 = gtimer();
      while (!mbar_try_wait(q_full, 0) && gtimer() - t0 < kWaitNs) {}
      for (int s = 0; s < NST; s++)
        if (issued[s]) {
          t0 = gtimer();
          while (!mbar_try_wait(&kv_full[s], iph[s]) && gtimer() - t0 < kWaitNs) {}
        }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_s = idesc_f16<T, TK>();
      const uint32_t id_pv = idesc_f16<T, HD, 128, true>();
      bool ok = mbar_wait(q_full, 0, abort, &g_attn_err);
      int pv_issued = 0;
      for (int j = 0; ok && j <= nb; j++) {
        if (j < nb) {
          const int st = j % NST;
          if (!mbar_wait(&kv_full[st], (j / NST) & 1, abort, &g_attn_err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d = tmem + (uint32_t)((j & 1) * TK);
          const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK + st * KV_BYTES);
#pragma unroll
          for (int kk = 0; kk < HD / 16; kk++) tc_mma(d, sdesc_sw128(qa + kk * 32), sdesc_sw128(ka + kk * 32), id_s, kk > 0 ? 1u : 0u);
          tc_commit(&s_full[j & 1]);
        }
        if (j >= 1) {
          const int jj = j - 1, b = jj & 1;
          if (!mbar_wait(&p_ready[b], (jj >> 1) & 1, abort, &g_attn_err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t va = smem_u32(sV + (jj % NST) * KV_BYTES);
#pragma unroll
          for (int kk = 0; kk < TK / 16; kk++)
            tc_mma_ts(tmem + o_col, tmem + (uint32_t)(b * TK + kk * 8), sdesc_sw128_mn(va + kk * 2048), id_pv, (jj > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&o_done[jj & 1]);
          tc_commit(&kv_empty[jj % NST]);
          pv_issued++;
        }
      }
      if (pv_issued) {  // the MMAs issued here finish before TMEM is freed
        const int last = pv_issued - 1;
        uint64_t t0 = gtimer();
        while (!mbar_try_wait(&o_done[last & 1], (last >> 1) & 1) && gtimer() - t0 < kWaitNs) {}
      }
    }
  } else {
    // softmax / correction / epilogue: thread <-> query row
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int qi = q0 + row;
    const int qw = q0 + quarter * 32;  // first query row of this warp
    const bool warp_live = qw < L;     // warps wholly past the sequence end skip their exps
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nb; j++) {
      const int b = j & 1;
      if (!mbar_wait(&s_full[b], (j >> 1) & 1, abort, &g_attn_err)) { ok = false; break; }
      tc_fence_after();
      const int kbase = kv_lo + j * TK;
      // this row's visible keys, relative to the block: [lo, hi]
      const int lo = (LOCAL ? max(0, qi - a.half_window) : 0) - kbase;
      const int hi = (LOCAL ? min(L - 1, qi + a.half_window) : L - 1) - kbase;
      // per 32-key chunk, warp-uniform: live = some row sees a key of it; full = every row sees all of it
      bool live[TK / 32], full[TK / 32];
#pragma unroll
      for (int c = 0; c < TK / 32; c++) {
        const int c0 = c * 32, c1 = c0 + 31;
        live[c] = warp_live && __any_sync(0xffffffffu, c1 >= lo && c0 <= hi);
        full[c] = __all_sync(0xffffffffu, c0 >= lo && c1 <= hi);
      }
      float s[TK];
      {
        uint32_t sr[TK];
#pragma unroll
        for (int c = 0; c < TK / 32; c++)
          if (live[c]) tmem_ld32(tmem + lane_off + (uint32_t)(b * TK + c * 32), sr + c * 32);
        tmem_wait_ld();  // one wait for every load issued above
#pragma unroll
        for (int i = 0; i < TK; i++) s[i] = __uint_as_float(sr[i]);
      }
      // row max of the raw scores (the softmax scale is positive, so it commutes)
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < TK / 32; c++) {
        if (!live[c]) continue;
        if (full[c]) {
#pragma unroll
          for (int i = 0; i < 32; i++) mx = fmaxf(mx, s[c * 32 + i]);
        } else {
#pragma unroll
          for (int i = 0; i < 32; i++) {
            const int k = c * 32 + i;
            const float v = (k >= lo && k <= hi) ? s[k] : -INFINITY;
            s[k] = v;
            mx = fmaxf(mx, v);
          }
        }
      }
      // lazy rescale: the reference max (raw units) only moves when it grew by more
      // than 2^8 after scaling, so P stays below 256 and O needs rescaling rarely
      const float sl = a.scale_log2;
      const float m_new = fmaxf(m, mx);
      const bool grow = (m_new - m) * sl > 8.f;  // m = -inf: true unless the row is still all masked
      const float corr = grow ? ex2((m - m_new) * sl) : 1.f;
      if (grow) m = m_new;
      const float nbias = m == -INFINITY ? 0.f : -m * sl;
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < TK / 32; c++) {
#pragma unroll
        for (int i = 0; i < 32; i++) {
          float p = 0.f;
          if (live[c]) p = ex2(fmaf(s[c * 32 + i], sl, nbias));
          s[c * 32 + i] = p;
          rs += p;
        }
      }
      l = l * corr + rs;
#pragma unroll
      for (int c = 0; c < TK / 64; c++) {
        uint32_t pr[32];
#pragma unroll
        for (int i = 0; i < 32; i++) pr[i] = pack2<T>(s[c * 64 + 2 * i], s[c * 64 + 2 * i + 1]);
        tmem_st32(tmem + lane_off + (uint32_t)(b * TK + c * 32), pr);
      }
      tmem_wait_st();
      if (j >= 1 && __any_sync(0xffffffffu, grow)) {
        // O holds blocks < j once P_{j-1}·V_{j-1} is done; rescale it before P_j·V_j
        if (!mbar_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, abort, &g_attn_err)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < HD / 32; c++) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_off + o_col + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; i++) r[i] = __float_as_uint(__uint_as_float(r[i]) * corr);
          tmem_st32(tmem + lane_off + o_col + c * 32, r);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[b]);
    }
    if (ok && mbar_wait(&o_done[(nb - 1) & 1], ((nb - 1) >> 1) & 1, abort, &g_attn_err)) {
      tc_fence_after();
      const float inv = 1.f / l;
      T* out = (T*)a.out + ((int64_t)tok0 + qi) * a.H + h * HD;
#pragma unroll
      for (int c = 0; c < HD / 32; c++) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + o_col + c * 32, r);
        tmem_wait_ld();
        if (qi < L) {
#pragma unroll
          for (int q = 0; q < 4; q++) {
            uint4 v;
            uint32_t* pv = (uint32_t*)&v;
#pragma unroll
            for (int i = 0; i < 4; i++)
              pv[i] = pack2<T>(__uint_as_float(r[q * 8 + 2 * i]) * inv, __uint_as_float(r[q * 8 + 2 * i + 1]) * inv);
            *(uint4*)(out + c * 32 + q * 8) = v;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

template <typename T, bool LOCAL>
void launch_attn(const CUtensorMap& mq, const CUtensorMap& mkv, const AttnTcArgs& a, int ntiles, int heads, cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    CUDA_OK(cudaFuncSetAttribute(k_attn_tc<T, LOCAL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ATTN_SMEM));
    attr = true;
  }
  k_attn_tc<T, LOCAL><<<dim3((unsigned)ntiles, (unsigned)heads), 192, ATTN_SMEM, st>>>(mq, mkv, a);
}

}  // namespace

namespace lc {

// Tile list for the tcgen05 kernel: one entry per 128-row query tile.
std::vector<int4> attention_tiles_tc(const int32_t* cu, int nseq) {
  std::vector<int4> t;
  for (int s = 0; s < nseq; s++) {
    int L = cu[s + 1] - cu[s];
    for (int q0 = 0; q0 < L; q0 += TQ) t.push_back(make_int4(cu[s], L, q0, 0));
  }
  return t;
}

void attention_varlen_tc(const void* qkv, void* out, const int4* tiles_dev, int ntiles, int64_t T, int H, int half_window, float scale,
                         int dtype, cudaStream_t st) {
  LC_CHECK(H % HD == 0 && T < INT32_MAX, "attention: head dim must be 64");
  if (ntiles == 0) return;
  LC_CHECK(ntiles < (1 << 30), "attention: too many tiles");
  const CUtensorMap& mq = tensor_map_2d(qkv, T, 3 * (int64_t)H, 3 * (int64_t)H, 64, TQ, dtype);
  const CUtensorMap& mkv = tensor_map_2d(qkv, T, 3 * (int64_t)H, 3 * (int64_t)H, 64, TK, dtype);
  AttnTcArgs a{tiles_dev, out, H, half_window, scale * 1.4426950408889634f};
  const int heads = H / HD;
  if (dtype == LC_F16) {
    if (half_window >= 0) launch_attn<__half, true>(mq, mkv, a, ntiles, heads, st);
    else launch_attn<__half, false>(mq, mkv, a, ntiles, heads, st);
  } else {
    if (half_window >= 0) launch_attn<__nv_bfloat16, true>(mq, mkv, a, ntiles, heads, st);
    else launch_attn<__nv_bfloat16, false>(mq, mkv, a, ntiles, heads, st);
  }
  LC_LAUNCHED(1);
}

std::string take_attention_errors() {
  unsigned int e = 0, z = 0;
  CUDA_OK(cudaMemcpyFromSymbol(&e, g_attn_err, sizeof(e)));
  if (!e) return "";
  CUDA_OK(cudaMemcpyToSymbol(g_attn_err, &z, sizeof(z)));
  return "tcgen05 attention: a pipeline wait timed out (kernel aborted its tile)";
}

}  // namespace lc
