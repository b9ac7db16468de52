// CPU restatement of the ModernBERT encoder forward and its CLS classifier
// head, in C++ — TEST INFRASTRUCTURE and the timed CPU baseline only: the
// product path (laya_js_b200) never loads, calls or links this file.
//
// Numerics follow the reference's CPU backend as the contract documents it
// ("f32 reference backend ... over packed f64 panels",
// packages/backend-cpu/README.md:37-39): every tensor is stored in f32, every
// op computes in f64 and rounds its result once to f32. Op for op this is the
// same restatement as oracle/ops.py, which the reference's golden vectors pin
// (tests/test_oracle_golden.py); tests/test_oracle_cpu.py pins this file to
// those vectors and to oracle/models.py.
//
//   linear      packages/tensor-backend/src/index.ts:211-215 (y = x·wᵀ + b)
//   layerNorm   index.ts:216-217 (biased variance, weight only for ModernBERT)
//   rope        index.ts:225-229 with MLX's f32 angle rule,
//               packages/backend-webgpu/src/backend.ts:1179-1195
//   sdpa        index.ts:230-237 (bool mask; here the window rule of
//               packages/modernbert/src/index.ts:240-259 on unpadded sequences)
//   geglu       packages/tensor-backend/src/compose.ts:87-93
//   encoder     packages/modernbert/src/index.ts:336-429 (embeddings :336-339,
//               layer :342-357, finalNorm :359-362)
//   head        softmax(linear(CLS row)), the op pattern of packages/laya/src/model.ts:228
//
// The weights of each Linear are packed once into f64 panels of 8 output
// rows interleaved along K, so the GEMM's inner loop streams one panel and
// keeps a 4 x 8 block of f64 accumulators in registers. Threads: std::thread
// workers over static or dynamic index ranges, the count given per call
// (1 = the single-threaded analogue of backend-cpu).
#include <immintrin.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <thread>
#include <chrono>
#include <cmath>
#include <cstring>
#include <vector>

namespace {

// f(i) for i in [0, n) on `threads` threads: contiguous chunks, or one index at
// a time from a shared counter when the items differ in cost.
template <class F>
void parallel_for(int64_t n, int threads, F&& f, bool dynamic = false) {
  const int T = (int)std::max<int64_t>(1, std::min<int64_t>(threads, n));
  if (T == 1) {
    for (int64_t i = 0; i < n; ++i) f(i);
    return;
  }
  std::atomic<int64_t> next{0};
  auto work = [&](int tid) {
    if (dynamic) {
      for (int64_t i = next++; i < n; i = next++) f(i);
    } else {
      const int64_t a = n * tid / T, b = n * (tid + 1) / T;
      for (int64_t i = a; i < b; ++i) f(i);
    }
  };
  std::vector<std::thread> ts;
  ts.reserve((size_t)T - 1);
  for (int t = 1; t < T; ++t) ts.emplace_back(work, t);
  work(0);
  for (auto& t : ts) t.join();
}

constexpr int PW = 8;  // output rows per packed panel
constexpr int MR = 4;  // x rows per register block

struct Panel {
  int64_t N = 0, K = 0;
  std::vector<double> p;  // [ceil(N/8)][K][8]
  void pack(const float* w, int64_t n, int64_t k) {
    N = n;
    K = k;
    int64_t np = (n + PW - 1) / PW;
    p.assign((size_t)(np * k * PW), 0.0);
    for (int64_t r = 0; r < n; ++r)
      for (int64_t j = 0; j < k; ++j) p[(size_t)(((r / PW) * k + j) * PW + r % PW)] = (double)w[r * k + j];
  }
};

// y[M, N] = f32(x[M, K] · wᵀ (+ b)), x already widened to f64. Work items are
// blocks of 64 rows x 8 panels (64 output columns), so a block's rows and
// panels stay in the core's L2 while the 4 x 8 register blocks walk them.
void gemm(const double* x, int64_t M, const Panel& w, const float* bias, float* y, int threads) {
  constexpr int64_t MC = 64, NG = 8;
  const int64_t K = w.K, N = w.N, np = (N + PW - 1) / PW;
  const int64_t mcs = (M + MC - 1) / MC, ngs = (np + NG - 1) / NG;
  parallel_for(mcs * ngs, threads, [&](int64_t job) {
    const int64_t mc = job / ngs, g = job % ngs;
    for (int64_t pj = g * NG; pj < std::min(np, (g + 1) * NG); ++pj) {
      const double* pp = w.p.data() + (size_t)(pj * K * PW);
      for (int64_t i0 = mc * MC; i0 < std::min(M, (mc + 1) * MC); i0 += MR) {
        const double* x0 = x + std::min(i0 + 0, M - 1) * K;
        const double* x1 = x + std::min(i0 + 1, M - 1) * K;
        const double* x2 = x + std::min(i0 + 2, M - 1) * K;
        const double* x3 = x + std::min(i0 + 3, M - 1) * K;
        __m256d a00 = _mm256_setzero_pd(), a01 = a00, a10 = a00, a11 = a00, a20 = a00, a21 = a00, a30 = a00, a31 = a00;
        for (int64_t k = 0; k < K; ++k) {
          const __m256d w0 = _mm256_loadu_pd(pp + k * PW), w1 = _mm256_loadu_pd(pp + k * PW + 4);
          __m256d b = _mm256_broadcast_sd(x0 + k);
          a00 = _mm256_fmadd_pd(b, w0, a00);
          a01 = _mm256_fmadd_pd(b, w1, a01);
          b = _mm256_broadcast_sd(x1 + k);
          a10 = _mm256_fmadd_pd(b, w0, a10);
          a11 = _mm256_fmadd_pd(b, w1, a11);
          b = _mm256_broadcast_sd(x2 + k);
          a20 = _mm256_fmadd_pd(b, w0, a20);
          a21 = _mm256_fmadd_pd(b, w1, a21);
          b = _mm256_broadcast_sd(x3 + k);
          a30 = _mm256_fmadd_pd(b, w0, a30);
          a31 = _mm256_fmadd_pd(b, w1, a31);
        }
        double acc[MR][PW];
        _mm256_storeu_pd(acc[0], a00);
        _mm256_storeu_pd(acc[0] + 4, a01);
        _mm256_storeu_pd(acc[1], a10);
        _mm256_storeu_pd(acc[1] + 4, a11);
        _mm256_storeu_pd(acc[2], a20);
        _mm256_storeu_pd(acc[2] + 4, a21);
        _mm256_storeu_pd(acc[3], a30);
        _mm256_storeu_pd(acc[3] + 4, a31);
        for (int r = 0; r < MR; ++r) {
          const int64_t i = i0 + r;
          if (i >= M) break;
          for (int c = 0; c < PW; ++c) {
            const int64_t n = pj * PW + c;
            if (n >= N) break;
            y[i * N + n] = (float)(acc[r][c] + (bias ? (double)bias[n] : 0.0));
          }
        }
      }
    }
  });
}

void widen(const float* a, int64_t n, std::vector<double>& out, int threads) {
  out.resize((size_t)n);
  double* o = out.data();
  parallel_for((n + 4095) / 4096, threads, [&](int64_t c) {
    for (int64_t i = c * 4096, e = std::min(n, i + 4096); i < e; ++i) o[i] = (double)a[i];
  });
}

void layer_norm(const float* x, int64_t rows, int64_t H, const float* w, const float* b, double eps, float* y, int threads) {
  parallel_for(rows, threads, [&](int64_t r) {
    const float* xr = x + r * H;
    double mu = 0.0;
    for (int64_t j = 0; j < H; ++j) mu += (double)xr[j];
    mu /= (double)H;
    double var = 0.0;
    for (int64_t j = 0; j < H; ++j) {
      const double d = (double)xr[j] - mu;
      var += d * d;
    }
    var /= (double)H;
    const double inv = std::sqrt(var + eps);
    for (int64_t j = 0; j < H; ++j) {
      double v = ((double)xr[j] - mu) / inv;
      if (w) v *= (double)w[j];
      if (b) v += (double)b[j];
      y[r * H + j] = (float)v;
    }
  });
}

// cos/sin [L][D/2] with the f32 angle rounding of MLX (backend.ts:1179-1195).
void rope_tables(int64_t L, int64_t D, double base, std::vector<double>& cs, std::vector<double>& sn) {
  const int64_t half = D / 2;
  const float lb = (float)std::log2(base);
  cs.resize((size_t)(L * half));
  sn.resize((size_t)(L * half));
  for (int64_t i = 0; i < half; ++i) {
    const float e = (float)(-(double)(float)((double)i / (double)half) * (double)lb);
    const float inv = (float)std::pow(2.0, (double)e);
    for (int64_t l = 0; l < L; ++l) {
      const float th = (float)((double)l * (double)inv);
      cs[(size_t)(l * half + i)] = std::cos((double)th);
      sn[(size_t)(l * half + i)] = std::sin((double)th);
    }
  }
}

inline double gelu(double v) { return 0.5 * v * (1.0 + std::erf(v / std::sqrt(2.0))); }

// Σ_d a[d]·b[d] over f32 rows, in f64 (four partial sums of four lanes).
inline double dot_f64(const float* a, const float* b, int64_t D) {
  __m256d s = _mm256_setzero_pd();
  int64_t d = 0;
  for (; d + 4 <= D; d += 4) s = _mm256_fmadd_pd(_mm256_cvtps_pd(_mm_loadu_ps(a + d)), _mm256_cvtps_pd(_mm_loadu_ps(b + d)), s);
  double lanes[4];
  _mm256_storeu_pd(lanes, s);
  double r = (lanes[0] + lanes[1]) + (lanes[2] + lanes[3]);
  for (; d < D; ++d) r += (double)a[d] * (double)b[d];
  return r;
}

// One (sequence, head) of attention. q, k, v: rows of `ld` floats starting at
// the head's column; positions 0..L-1; keys visible to query i: all when
// half_window < 0, else |i − j| <= half_window. out: rows of `ldo` floats.
// D <= 256.
void attend(const float* q, const float* k, const float* v, int64_t ld, int64_t L, int64_t D, double scale, int64_t half_window,
            float* out, int64_t ldo, std::vector<double>& s) {
  s.resize((size_t)L);
  double o[256];
  for (int64_t i = 0; i < L; ++i) {
    const int64_t j0 = half_window < 0 ? 0 : std::max<int64_t>(0, i - half_window);
    const int64_t j1 = half_window < 0 ? L : std::min<int64_t>(L, i + half_window + 1);
    double m = -INFINITY;
    for (int64_t j = j0; j < j1; ++j) {
      const double a = dot_f64(q + i * ld, k + j * ld, D) * scale;
      s[(size_t)j] = a;
      m = std::max(m, a);
    }
    double z = 0.0;
    for (int64_t j = j0; j < j1; ++j) {
      s[(size_t)j] = std::exp(s[(size_t)j] - m);
      z += s[(size_t)j];
    }
    for (int64_t d = 0; d < D; ++d) o[d] = 0.0;
    for (int64_t j = j0; j < j1; ++j) {
      const double p = s[(size_t)j] / z;
      const float* vr = v + j * ld;
      for (int64_t d = 0; d < D; ++d) o[d] += p * (double)vr[d];
    }
    for (int64_t d = 0; d < D; ++d) out[i * ldo + d] = (float)o[d];
  }
}

struct Layer {
  std::vector<float> attn_norm, mlp_norm;
  Panel wqkv, wo, wi, wmo;
  bool global = false;
};

struct Encoder {
  int64_t V, H, I, nl, nh, window;
  double eps, theta_g, theta_l;
  std::vector<float> tok, emb_norm, final_norm;
  std::vector<Layer> layers;
  std::vector<double> cos_g, sin_g, cos_l, sin_l;
  int64_t rope_len = 0;

  void ensure_rope(int64_t L) {
    if (L <= rope_len) return;
    rope_tables(L, H / nh, theta_g, cos_g, sin_g);
    rope_tables(L, H / nh, theta_l, cos_l, sin_l);
    rope_len = L;
  }
};

}  // namespace

extern "C" {

// icfg: vocab, hidden, intermediate, layers, heads, local_attention, global_every.
// dcfg: norm_eps, rope_theta_global, rope_theta_local.
// w: tok [V,H], emb_norm [H]; per layer: attn_norm [H] (null for layer 0),
// Wqkv [3H,H], Wo [H,H], mlp_norm [H], Wi [2I,H], mlp.Wo [H,I]; final_norm [H].
void* oc_encoder_create(const int32_t* icfg, const double* dcfg, const float* const* w, int nw) {
  auto* e = new Encoder();
  e->V = icfg[0];
  e->H = icfg[1];
  e->I = icfg[2];
  e->nl = icfg[3];
  e->nh = icfg[4];
  e->window = icfg[5];
  const int every = icfg[6];
  e->eps = dcfg[0];
  e->theta_g = dcfg[1];
  e->theta_l = dcfg[2];
  if (nw != 3 + 6 * e->nl) {
    delete e;
    return nullptr;
  }
  const int64_t H = e->H, I = e->I;
  int at = 0;
  e->tok.assign(w[at], w[at] + e->V * H);
  ++at;
  e->emb_norm.assign(w[at], w[at] + H);
  ++at;
  e->layers.resize((size_t)e->nl);
  for (int64_t i = 0; i < e->nl; ++i) {
    Layer& L = e->layers[(size_t)i];
    L.global = (i % every) == 0;
    if (w[at]) L.attn_norm.assign(w[at], w[at] + H);
    ++at;
    L.wqkv.pack(w[at++], 3 * H, H);
    L.wo.pack(w[at++], H, H);
    L.mlp_norm.assign(w[at], w[at] + H);
    ++at;
    L.wi.pack(w[at++], 2 * I, H);
    L.wmo.pack(w[at++], H, I);
  }
  e->final_norm.assign(w[at], w[at] + H);
  return e;
}

void oc_encoder_free(void* p) { delete static_cast<Encoder*>(p); }

// ids [T] packed, cu [nseq + 1]; head_w [C, H] and head_b [C] (f32, may be
// null when C == 0); probs [nseq, C]; hidden [T, H] final-norm states (may be
// null). Returns the wall seconds of the forward (host clock).
double oc_encoder_forward(void* p, const int32_t* ids, const int32_t* cu, int nseq, const float* head_w, const float* head_b, int C,
                          float* probs, float* hidden, int threads) {
  auto t0 = std::chrono::steady_clock::now();
  Encoder& e = *static_cast<Encoder*>(p);
  const int64_t T = cu[nseq], H = e.H, I = e.I, nh = e.nh, hd = H / nh, half = hd / 2;
  int64_t Lmax = 0;
  for (int s = 0; s < nseq; ++s) Lmax = std::max<int64_t>(Lmax, cu[s + 1] - cu[s]);
  e.ensure_rope(Lmax);
  std::vector<float> x((size_t)(T * H)), h((size_t)(T * H)), qkv((size_t)(T * 3 * H)), att((size_t)(T * H)), t1((size_t)(T * H)),
      m((size_t)(T * 2 * I)), g((size_t)(T * I));
  std::vector<double> xd;
  // embeddings: LayerNorm(tok[ids])
  parallel_for(T, threads, [&](int64_t t) { std::memcpy(&h[(size_t)(t * H)], &e.tok[(size_t)((int64_t)ids[t] * H)], (size_t)H * sizeof(float)); });
  layer_norm(h.data(), T, H, e.emb_norm.data(), nullptr, e.eps, x.data(), threads);
  const double scale = 1.0 / std::sqrt((double)hd);
  for (int64_t li = 0; li < e.nl; ++li) {
    Layer& L = e.layers[(size_t)li];
    const float* hin = x.data();
    if (!L.attn_norm.empty()) {
      layer_norm(x.data(), T, H, L.attn_norm.data(), nullptr, e.eps, h.data(), threads);
      hin = h.data();
    }
    widen(hin, T * H, xd, threads);
    gemm(xd.data(), T, L.wqkv, nullptr, qkv.data(), threads);
    // RoPE on q and k (rows [L, 3, nh, hd]), rounded to f32 like the op's output
    const std::vector<double>& cs = L.global ? e.cos_g : e.cos_l;
    const std::vector<double>& sn = L.global ? e.sin_g : e.sin_l;
    parallel_for(nseq, threads, [&](int64_t s) {
      for (int64_t t = cu[s]; t < cu[s + 1]; ++t) {
        const int64_t pos = t - cu[s];
        for (int64_t part = 0; part < 2; ++part)
          for (int64_t hh = 0; hh < nh; ++hh) {
            float* r = &qkv[(size_t)(t * 3 * H + part * H + hh * hd)];
            for (int64_t i = 0; i < half; ++i) {
              const double a = r[i], b = r[i + half], c = cs[(size_t)(pos * half + i)], sv = sn[(size_t)(pos * half + i)];
              r[i] = (float)(a * c - b * sv);
              r[i + half] = (float)(b * c + a * sv);
            }
          }
      }
    });
    const int64_t hw = L.global ? -1 : e.window / 2;
    parallel_for((int64_t)nseq * nh, threads, [&](int64_t job) {
      thread_local std::vector<double> sbuf;
      const int64_t s = job / nh, hh = job % nh;
      const int64_t t0s = cu[s], Ls = cu[s + 1] - cu[s];
      const float* base = &qkv[(size_t)(t0s * 3 * H + hh * hd)];
      attend(base, base + H, base + 2 * H, 3 * H, Ls, hd, scale, hw, &att[(size_t)(t0s * H + hh * hd)], H, sbuf);
    }, true);
    widen(att.data(), T * H, xd, threads);
    gemm(xd.data(), T, L.wo, nullptr, t1.data(), threads);
    parallel_for(T, threads, [&](int64_t t) {
      for (int64_t i = t * H; i < (t + 1) * H; ++i) x[(size_t)i] = (float)((double)x[(size_t)i] + (double)t1[(size_t)i]);
    });
    layer_norm(x.data(), T, H, L.mlp_norm.data(), nullptr, e.eps, h.data(), threads);
    widen(h.data(), T * H, xd, threads);
    gemm(xd.data(), T, L.wi, nullptr, m.data(), threads);
    parallel_for(T, threads, [&](int64_t t) {
      for (int64_t j = 0; j < I; ++j)
        g[(size_t)(t * I + j)] = (float)(gelu((double)m[(size_t)(t * 2 * I + j)]) * (double)m[(size_t)(t * 2 * I + I + j)]);
    });
    widen(g.data(), T * I, xd, threads);
    gemm(xd.data(), T, L.wmo, nullptr, t1.data(), threads);
    parallel_for(T, threads, [&](int64_t t) {
      for (int64_t i = t * H; i < (t + 1) * H; ++i) x[(size_t)i] = (float)((double)x[(size_t)i] + (double)t1[(size_t)i]);
    });
  }
  float* out = hidden ? hidden : h.data();
  layer_norm(x.data(), T, H, e.final_norm.data(), nullptr, e.eps, out, threads);
  if (C > 0 && probs) {
    for (int s = 0; s < nseq; ++s) {
      const float* cls = out + (int64_t)cu[s] * H;
      std::vector<float> z((size_t)C);
      for (int c = 0; c < C; ++c) {
        double a = 0.0;
        for (int64_t j = 0; j < H; ++j) a += (double)cls[j] * (double)head_w[c * H + j];
        z[(size_t)c] = (float)(a + (head_b ? (double)head_b[c] : 0.0));
      }
      double mx = -INFINITY, sum = 0.0;
      for (int c = 0; c < C; ++c) mx = std::max(mx, (double)z[(size_t)c]);
      for (int c = 0; c < C; ++c) sum += std::exp((double)z[(size_t)c] - mx);
      for (int c = 0; c < C; ++c) probs[s * C + c] = (float)(std::exp((double)z[(size_t)c] - mx) / sum);
    }
  }
  return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

// ---- single ops, for pinning this file to the reference's golden vectors

void oc_linear(const float* x, int64_t M, int64_t K, const float* w, int64_t N, const float* b, float* y, int threads) {
  Panel p;
  p.pack(w, N, K);
  std::vector<double> xd;
  widen(x, M * K, xd, threads);
  gemm(xd.data(), M, p, b, y, threads);
}

void oc_layer_norm(const float* x, int64_t rows, int64_t H, const float* w, const float* b, double eps, float* y) {
  layer_norm(x, rows, H, w, b, eps, y, 1);
}

// x [outer, L, D] → y, positions 0..L-1.
void oc_rope(const float* x, int64_t outer, int64_t L, int64_t D, double base, float* y) {
  std::vector<double> cs, sn;
  rope_tables(L, D, base, cs, sn);
  const int64_t half = D / 2;
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t l = 0; l < L; ++l) {
      const float* r = x + (o * L + l) * D;
      float* w = y + (o * L + l) * D;
      for (int64_t i = 0; i < half; ++i) {
        const double a = r[i], b = r[i + half], c = cs[(size_t)(l * half + i)], s = sn[(size_t)(l * half + i)];
        w[i] = (float)(a * c - b * s);
        w[i + half] = (float)(b * c + a * s);
      }
    }
}

// q [BH, Lq, D], k [BH, Lk, D], v [BH, Lk, Dv], mask [BH, Lq, Lk] bytes or null.
void oc_sdpa(const float* q, const float* k, const float* v, const uint8_t* mask, int64_t BH, int64_t Lq, int64_t Lk, int64_t D,
             int64_t Dv, double scale, float* out) {
  std::vector<double> s((size_t)Lk);
  for (int64_t b = 0; b < BH; ++b)
    for (int64_t i = 0; i < Lq; ++i) {
      double m = -INFINITY;
      for (int64_t j = 0; j < Lk; ++j) {
        double a = 0.0;
        for (int64_t d = 0; d < D; ++d) a += (double)q[(b * Lq + i) * D + d] * (double)k[(b * Lk + j) * D + d];
        a *= scale;
        if (mask && !mask[(b * Lq + i) * Lk + j]) a = -INFINITY;
        s[(size_t)j] = a;
        m = std::max(m, a);
      }
      double z = 0.0;
      for (int64_t j = 0; j < Lk; ++j) {
        s[(size_t)j] = std::exp(s[(size_t)j] - m);
        z += s[(size_t)j];
      }
      for (int64_t d = 0; d < Dv; ++d) {
        double o = 0.0;
        for (int64_t j = 0; j < Lk; ++j) o += (s[(size_t)j] / z) * (double)v[(b * Lk + j) * Dv + d];
        out[(b * Lq + i) * Dv + d] = (float)o;
      }
    }
}

// x [rows, 2F] → gelu(x[:, :F]) · x[:, F:]
void oc_geglu(const float* x, int64_t rows, int64_t F, float* y) {
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t j = 0; j < F; ++j) y[r * F + j] = (float)(gelu((double)x[r * 2 * F + j]) * (double)x[r * 2 * F + F + j]);
}

}  // extern "C"
