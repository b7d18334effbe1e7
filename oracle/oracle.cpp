// CPU F32 restatement of the Vestra Engine DA3 ViT attention sub-block.
//
// TEST INFRASTRUCTURE ONLY.  Nothing in the product path links, loads or calls
// this file: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
// leg do, and only as the checker / the timed CPU baseline.
//
// Why a restatement: the reference's arithmetic lives in the external crate
// `vestra-kernels` (git rev 783bd66cb22ff019ec6bbad0f9b8eb1632a6a14f, pinned in
// the reference's Cargo.toml:27 / Cargo.lock:1784-1786), which is not vendored,
// and there is no Rust toolchain here.  This file restates the semantics the
// reference's own call sites define:
//
//   * crates/da-engine/src/vit_block.rs:772-992   run_attention (QKV -> head split
//     -> gated QK-LayerNorm -> gated 2D RoPE -> SDPA core -> unpack -> proj [* ls1])
//   * crates/da-engine/src/vit_block.rs:841-881   RoPE position table
//   * crates/da-engine/src/vit_block.rs:686       QK_NORM_EPS = 1e-5
//   * crates/da-engine/src/vit_block.rs:721-761   run_linear (bias, presence-gated ls1)
//   * crates/da-graph/src/cpu_backend.rs:198-298  Op::Attention (LN over heads*n rows
//     of head_dim, then rope2d on q and k with rounded positions, then attention)
//   * docs/plans/2026-07-18-rust-engine-v1.md:1290  RoPE: head_dim split into a y half
//     and an x half, rotary per half, base frequency 100.
//
// Parity status: the attention, LayerNorm, projection and position semantics are
// pinned by the reference's relation tests (restated in tests/test_oracle.py).  The
// RoPE pairing inside each half (rotate-half, pairs (i, i+h/2)) is NOT pinned: the
// only golden vector for it (`rope_out` in the reference's dump file) is absent.
// `pairing` selects between rotate-half (0, default) and interleaved pairs (1).
//
// Build: oracle/Makefile (g++ -O3 -fopenmp).  AVX-512 paths are compiled with
// per-function target attributes and chosen at run time, so the same .so runs on
// hosts without AVX-512 (scalar fallback).

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <vector>

#include <immintrin.h>
#include <omp.h>

namespace {

bool have_avx512() {
  static int cached = -1;
  if (cached < 0) {
    __builtin_cpu_init();
    cached = (__builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
              __builtin_cpu_supports("avx512vl") && __builtin_cpu_supports("fma"))
                 ? 1
                 : 0;
  }
  return cached == 1;
}

int resolve_threads(int threads) { return threads > 0 ? threads : omp_get_max_threads(); }

// ---------------------------------------------------------------------------
// Row LayerNorm, torch nn.LayerNorm semantics (biased variance), as used for
// LN1 (vit_block.rs:696-714) and per-(head,token) QK-norm (cpu_backend.rs:251-275).
// ---------------------------------------------------------------------------
void layernorm_rows(float* x, int64_t rows, int cols, const float* g, const float* b, float eps,
                    int threads) {
#pragma omp parallel for num_threads(threads) schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    float* row = x + r * cols;
    double mean = 0.0;
    for (int c = 0; c < cols; ++c) mean += row[c];
    mean /= cols;
    double var = 0.0;
    for (int c = 0; c < cols; ++c) {
      double d = row[c] - mean;
      var += d * d;
    }
    var /= cols;
    const float inv = (float)(1.0 / std::sqrt(var + (double)eps));
    const float m = (float)mean;
    for (int c = 0; c < cols; ++c) row[c] = (row[c] - m) * inv * g[c] + b[c];
  }
}

// ---------------------------------------------------------------------------
// 2D RoPE on [heads, n, head_dim] (vestra_kernels::rope2d call sites:
// vit_block.rs:944-948, cpu_backend.rs:286-296).  The first head_dim/2 channels
// rotate with the y coordinate, the second half with x.  Within a half of width
// h, frequency i (i < h/2) is base^(-2i/h).  pairing 0 = rotate-half (channel i
// pairs with i + h/2); pairing 1 = interleaved (2i pairs with 2i+1).
// ---------------------------------------------------------------------------
void rope2d(float* x, int heads, int64_t n, int head_dim, const float* pos_yx, float base,
            int pairing, int threads) {
  const int half = head_dim / 2;
  const int nf = half / 2;
  std::vector<double> inv_freq(nf);
  for (int i = 0; i < nf; ++i) inv_freq[i] = std::pow((double)base, -(2.0 * i) / (double)half);
#pragma omp parallel for num_threads(threads) schedule(static)
  for (int64_t t = 0; t < n; ++t) {
    const double py = (double)std::llround(pos_yx[2 * t]);
    const double px = (double)std::llround(pos_yx[2 * t + 1]);
    for (int h = 0; h < heads; ++h) {
      float* row = x + ((int64_t)h * n + t) * head_dim;
      for (int axis = 0; axis < 2; ++axis) {
        float* seg = row + axis * half;
        const double p = axis == 0 ? py : px;
        for (int i = 0; i < nf; ++i) {
          const double ang = p * inv_freq[i];
          const float c = (float)std::cos(ang), s = (float)std::sin(ang);
          const int i0 = pairing == 0 ? i : 2 * i;
          const int i1 = pairing == 0 ? i + nf : 2 * i + 1;
          const float a = seg[i0], bb = seg[i1];
          seg[i0] = a * c - bb * s;
          seg[i1] = bb * c + a * s;
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// GEMM  C[M,N] = A[M,K] * B[K,N] (+ bias[N]) (* scale[N]), all row-major F32.
// B is the reference's [in,out] weight orientation (engine.rs:110-126).
// ---------------------------------------------------------------------------
__attribute__((target("avx512f,avx512vl,avx512bw,fma"))) void gemm_avx512(
    const float* A, int64_t M, int K, const float* B, int N, float* C, int threads) {
  // 4 rows x 32 columns register tile; K blocked for L1/L2 residency of the B panel.
  const int KB = 256;
  const int64_t mt = (M + 3) / 4;
  const int nt = N / 32;
#pragma omp parallel for num_threads(threads) collapse(2) schedule(static)
  for (int64_t bi = 0; bi < mt; ++bi) {
    for (int bj = 0; bj < nt; ++bj) {
      const int64_t i0 = bi * 4;
      const int rows = (int)std::min<int64_t>(4, M - i0);
      const int j0 = bj * 32;
      __m512 acc[4][2];
      for (int r = 0; r < 4; ++r) acc[r][0] = acc[r][1] = _mm512_setzero_ps();
      for (int k0 = 0; k0 < K; k0 += KB) {
        const int k1 = std::min(K, k0 + KB);
        for (int k = k0; k < k1; ++k) {
          const __m512 b0 = _mm512_loadu_ps(B + (int64_t)k * N + j0);
          const __m512 b1 = _mm512_loadu_ps(B + (int64_t)k * N + j0 + 16);
          for (int r = 0; r < rows; ++r) {
            const __m512 a = _mm512_set1_ps(A[(i0 + r) * K + k]);
            acc[r][0] = _mm512_fmadd_ps(a, b0, acc[r][0]);
            acc[r][1] = _mm512_fmadd_ps(a, b1, acc[r][1]);
          }
        }
      }
      for (int r = 0; r < rows; ++r) {
        _mm512_storeu_ps(C + (i0 + r) * N + j0, acc[r][0]);
        _mm512_storeu_ps(C + (i0 + r) * N + j0 + 16, acc[r][1]);
      }
    }
  }
  // Column tail (N not a multiple of 32): scalar.
  if (N % 32) {
    const int jt = (N / 32) * 32;
#pragma omp parallel for num_threads(threads) schedule(static)
    for (int64_t i = 0; i < M; ++i)
      for (int j = jt; j < N; ++j) {
        float s = 0.f;
        for (int k = 0; k < K; ++k) s += A[i * K + k] * B[(int64_t)k * N + j];
        C[i * N + j] = s;
      }
  }
}

void gemm_scalar(const float* A, int64_t M, int K, const float* B, int N, float* C, int threads) {
#pragma omp parallel for num_threads(threads) schedule(static)
  for (int64_t i = 0; i < M; ++i) {
    float* c = C + i * N;
    for (int j = 0; j < N; ++j) c[j] = 0.f;
    for (int k = 0; k < K; ++k) {
      const float a = A[i * K + k];
      const float* b = B + (int64_t)k * N;
      for (int j = 0; j < N; ++j) c[j] += a * b[j];
    }
  }
}

void linear(const float* A, int64_t M, int K, const float* B, int N, const float* bias,
            const float* scale, float* C, int threads) {
  if (have_avx512())
    gemm_avx512(A, M, K, B, N, C, threads);
  else
    gemm_scalar(A, M, K, B, N, C, threads);
  if (bias || scale) {
#pragma omp parallel for num_threads(threads) schedule(static)
    for (int64_t i = 0; i < M; ++i)
      for (int j = 0; j < N; ++j) {
        float v = C[i * N + j] + (bias ? bias[j] : 0.f);
        C[i * N + j] = scale ? v * scale[j] : v;
      }
  }
}

// ---------------------------------------------------------------------------
// Attention core: per head, softmax(Q K^T / sqrt(d)) V, non-causal, online
// softmax (vestra_kernels::attention at vit_block.rs:951-953).  The token axis
// is cut into independent segments of seg_len tokens: seg_len == n is one
// attention over all tokens (a single view, or a global block over the
// view-major flattened sequence); seg_len == tokens-per-view is the batch of
// local blocks, one attention per view.  q_rows (optional) restricts the
// computed query rows; out then holds [heads, nq, d] in q_rows order.
// ---------------------------------------------------------------------------

// exp(x) for the online softmax: Cody-Waite reduction by ln2 (hi/lo split) and a
// degree-6 Taylor polynomial on |f| <= ln2/2 (truncation error < 2e-7 relative);
// 2^n applied with vscalefps.  Inputs are <= 0 here; they are clamped at -87.
__attribute__((target("avx512f,avx512vl,avx512bw,fma"))) inline __m512 exp_avx512(__m512 x) {
  const __m512 log2e = _mm512_set1_ps(1.44269504088896341f);
  const __m512 ln2_hi = _mm512_set1_ps(0.693145751953125f);
  const __m512 ln2_lo = _mm512_set1_ps(1.42860682030941723e-6f);
  x = _mm512_max_ps(x, _mm512_set1_ps(-87.0f));
  const __m512 n = _mm512_roundscale_ps(_mm512_mul_ps(x, log2e),
                                        _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
  __m512 f = _mm512_fnmadd_ps(n, ln2_hi, x);
  f = _mm512_fnmadd_ps(n, ln2_lo, f);
  __m512 p = _mm512_set1_ps(1.0f / 720.0f);
  p = _mm512_fmadd_ps(p, f, _mm512_set1_ps(1.0f / 120.0f));
  p = _mm512_fmadd_ps(p, f, _mm512_set1_ps(1.0f / 24.0f));
  p = _mm512_fmadd_ps(p, f, _mm512_set1_ps(1.0f / 6.0f));
  p = _mm512_fmadd_ps(p, f, _mm512_set1_ps(0.5f));
  p = _mm512_fmadd_ps(p, f, _mm512_set1_ps(1.0f));
  p = _mm512_fmadd_ps(p, f, _mm512_set1_ps(1.0f));
  return _mm512_scalef_ps(p, n);
}

// Packs K of one head into d-major blocks of 32 keys: kt[blk][d][32], zero padded.
void pack_kt(const float* k, int64_t n, int d, std::vector<float>& kt) {
  const int64_t nb = (n + 31) / 32;
  kt.assign((size_t)(nb * d * 32), 0.f);
  for (int64_t t = 0; t < n; ++t) {
    const int64_t blk = t / 32, lane = t % 32;
    for (int c = 0; c < d; ++c) kt[(size_t)((blk * d + c) * 32 + lane)] = k[t * d + c];
  }
}

// One query tile of up to 4 rows against keys [k_begin, k_end) of one head, d == 64.
__attribute__((target("avx512f,avx512vl,avx512bw,fma"))) void attn_tile_avx512_d64(
    const float* const qrows[4], int nrows, const float* kt, const float* v, int64_t k_begin,
    int64_t k_end, float scale, float* const orow[4]) {
  const int D = 64;
  __m512 acc[4][4];
  float m[4], l[4];
  for (int r = 0; r < 4; ++r) {
    for (int c = 0; c < 4; ++c) acc[r][c] = _mm512_setzero_ps();
    m[r] = -std::numeric_limits<float>::infinity();
    l[r] = 0.f;
  }
  alignas(64) float p[4][32];
  // Keys are processed in 32-aligned blocks of the packed layout; keys outside
  // [k_begin, k_end) are masked off.
  for (int64_t blk = k_begin / 32; blk * 32 < k_end; ++blk) {
    const float* kb = kt + (size_t)blk * D * 32;
    __m512 s[4][2];
    for (int r = 0; r < 4; ++r) s[r][0] = s[r][1] = _mm512_setzero_ps();
    for (int c = 0; c < D; ++c) {
      const __m512 k0 = _mm512_loadu_ps(kb + c * 32);
      const __m512 k1 = _mm512_loadu_ps(kb + c * 32 + 16);
      for (int r = 0; r < nrows; ++r) {
        const __m512 qv = _mm512_set1_ps(qrows[r][c]);
        s[r][0] = _mm512_fmadd_ps(qv, k0, s[r][0]);
        s[r][1] = _mm512_fmadd_ps(qv, k1, s[r][1]);
      }
    }
    const int64_t t0 = blk * 32;
    uint32_t valid = 0;
    for (int j = 0; j < 32; ++j)
      if (t0 + j >= k_begin && t0 + j < k_end) valid |= 1u << j;
    const __mmask16 v0 = (__mmask16)(valid & 0xffff), v1 = (__mmask16)(valid >> 16);
    const __m512 ninf = _mm512_set1_ps(-std::numeric_limits<float>::infinity());
    for (int r = 0; r < nrows; ++r) {
      __m512 a = _mm512_mask_mul_ps(ninf, v0, s[r][0], _mm512_set1_ps(scale));
      __m512 b = _mm512_mask_mul_ps(ninf, v1, s[r][1], _mm512_set1_ps(scale));
      const float bm = _mm512_reduce_max_ps(_mm512_max_ps(a, b));
      const float mn = std::max(m[r], bm);
      const float alpha = (m[r] == -std::numeric_limits<float>::infinity())
                              ? 0.f
                              : (float)std::exp((double)(m[r] - mn));
      const __m512 mv = _mm512_set1_ps(mn);
      __m512 pa = _mm512_maskz_mov_ps(v0, exp_avx512(_mm512_sub_ps(a, mv)));
      __m512 pb = _mm512_maskz_mov_ps(v1, exp_avx512(_mm512_sub_ps(b, mv)));
      l[r] = l[r] * alpha + _mm512_reduce_add_ps(_mm512_add_ps(pa, pb));
      m[r] = mn;
      _mm512_store_ps(p[r], pa);
      _mm512_store_ps(p[r] + 16, pb);
      const __m512 al = _mm512_set1_ps(alpha);
      for (int c = 0; c < 4; ++c) acc[r][c] = _mm512_mul_ps(acc[r][c], al);
    }
    const int jlo = (int)std::max<int64_t>(0, k_begin - t0);
    const int jhi = (int)std::min<int64_t>(32, k_end - t0);
    for (int j = jlo; j < jhi; ++j) {
      const float* vr = v + (t0 + j) * D;
      const __m512 v0r = _mm512_loadu_ps(vr), v1r = _mm512_loadu_ps(vr + 16);
      const __m512 v2r = _mm512_loadu_ps(vr + 32), v3r = _mm512_loadu_ps(vr + 48);
      for (int r = 0; r < nrows; ++r) {
        const __m512 pv = _mm512_set1_ps(p[r][j]);
        acc[r][0] = _mm512_fmadd_ps(pv, v0r, acc[r][0]);
        acc[r][1] = _mm512_fmadd_ps(pv, v1r, acc[r][1]);
        acc[r][2] = _mm512_fmadd_ps(pv, v2r, acc[r][2]);
        acc[r][3] = _mm512_fmadd_ps(pv, v3r, acc[r][3]);
      }
    }
  }
  for (int r = 0; r < nrows; ++r) {
    const __m512 inv = _mm512_set1_ps(1.0f / l[r]);
    for (int c = 0; c < 4; ++c) _mm512_storeu_ps(orow[r] + 16 * c, _mm512_mul_ps(acc[r][c], inv));
  }
}

// Scalar online softmax for one query row (any head_dim).
void attn_row_scalar(const float* q, const float* k, const float* v, int64_t k_begin,
                     int64_t k_end, int d, float scale, float* o) {
  float m = -std::numeric_limits<float>::infinity(), l = 0.f;
  std::vector<float> acc(d, 0.f);
  for (int64_t t = k_begin; t < k_end; ++t) {
    float s = 0.f;
    for (int c = 0; c < d; ++c) s += q[c] * k[t * d + c];
    s *= scale;
    const float mn = std::max(m, s);
    const float alpha = std::exp(m - mn);
    const float p = std::exp(s - mn);
    l = l * alpha + p;
    for (int c = 0; c < d; ++c) acc[c] = acc[c] * alpha + p * v[t * d + c];
    m = mn;
  }
  for (int c = 0; c < d; ++c) o[c] = acc[c] / l;
}

void attention_core(const float* q, const float* k, const float* v, int heads, int64_t n, int d,
                    int64_t seg_len, const int64_t* q_rows, int64_t nq, float* out, int threads) {
  const float scale = 1.0f / std::sqrt((float)d);
  const bool fast = have_avx512() && d == 64;
  const int64_t nrows = q_rows ? nq : n;
  const int64_t tiles = (nrows + 3) / 4;
  for (int h = 0; h < heads; ++h) {
    const float* qh = q + (int64_t)h * n * d;
    const float* kh = k + (int64_t)h * n * d;
    const float* vh = v + (int64_t)h * n * d;
    float* oh = out + (int64_t)h * nrows * d;
    std::vector<float> kt;
    if (fast) pack_kt(kh, n, d, kt);
#pragma omp parallel for num_threads(threads) schedule(dynamic, 4)
    for (int64_t ti = 0; ti < tiles; ++ti) {
      // A tile holds up to 4 query rows that share one key segment.
      int64_t idx[4];
      int cnt = 0;
      for (int64_t i = ti * 4; i < std::min(nrows, ti * 4 + 4); ++i) idx[cnt++] = i;
      int64_t start = 0;
      while (start < cnt) {
        const int64_t t0 = q_rows ? q_rows[idx[start]] : idx[start];
        const int64_t seg = t0 / seg_len;
        int end = start + 1;
        while (end < cnt) {
          const int64_t te = q_rows ? q_rows[idx[end]] : idx[end];
          if (te / seg_len != seg) break;
          ++end;
        }
        const int64_t kb = seg * seg_len, ke = std::min(n, kb + seg_len);
        if (fast) {
          const float* qr[4] = {qh, qh, qh, qh};
          float* orow[4] = {nullptr, nullptr, nullptr, nullptr};
          alignas(64) float dummy[64];
          for (int r = 0; r < 4; ++r) {
            if (start + r < end) {
              const int64_t t = q_rows ? q_rows[idx[start + r]] : idx[start + r];
              qr[r] = qh + t * d;
              orow[r] = oh + idx[start + r] * d;
            } else {
              orow[r] = dummy;
            }
          }
          attn_tile_avx512_d64(qr, end - start, kt.data(), vh, kb, ke, scale, orow);
        } else {
          for (int r = start; r < end; ++r) {
            const int64_t t = q_rows ? q_rows[idx[r]] : idx[r];
            attn_row_scalar(qh + t * d, kh, vh, kb, ke, d, scale, oh + idx[r] * d);
          }
        }
        start = end;
      }
    }
  }
}

}  // namespace

extern "C" {

int oracle_has_avx512(void) { return have_avx512() ? 1 : 0; }

// RoPE position table (vit_block.rs:841-881; device-tail copy at :512-526).
// Special tokens (the first n_special of every view) get (0,0).  Patch p of a
// view gets (p/gw + 1, p%gw + 1) in local blocks and (1,1) in global blocks.
void oracle_positions(int64_t rows, int view_count, int n_special, int gh, int gw, int global,
                      float* pos_yx) {
  const int64_t per_view = (int64_t)n_special + (int64_t)gh * gw;
  std::memset(pos_yx, 0, sizeof(float) * 2 * rows);
  for (int v = 0; v < view_count; ++v)
    for (int64_t lt = n_special; lt < per_view; ++lt) {
      const int64_t t = v * per_view + lt;
      if (t >= rows) return;
      if (global) {
        pos_yx[2 * t] = 1.f;
        pos_yx[2 * t + 1] = 1.f;
      } else {
        const int64_t p = lt - n_special;
        pos_yx[2 * t] = (float)(p / gw + 1);
        pos_yx[2 * t + 1] = (float)(p % gw + 1);
      }
    }
}

void oracle_layernorm(float* x, int64_t rows, int cols, const float* g, const float* b, float eps,
                      int threads) {
  layernorm_rows(x, rows, cols, g, b, eps, resolve_threads(threads));
}

void oracle_rope2d(float* x, int heads, int64_t n, int head_dim, const float* pos_yx, float base,
                   int pairing, int threads) {
  rope2d(x, heads, n, head_dim, pos_yx, base, pairing, resolve_threads(threads));
}

void oracle_linear(const float* a, int64_t m, int k, const float* b, int n, const float* bias,
                   const float* scale, float* c, int threads) {
  linear(a, m, k, b, n, bias, scale, c, resolve_threads(threads));
}

// q, k, v, out: [heads, n, d].
void oracle_attention_core(const float* q, const float* k, const float* v, int heads, int64_t n,
                           int d, int64_t seg_len, float* out, int threads) {
  attention_core(q, k, v, heads, n, d, seg_len > 0 ? seg_len : n, nullptr, 0, out,
                 resolve_threads(threads));
}

// Op::Attention (graph.rs:67-105, cpu_backend.rs:198-298): optional per-(head,token)
// LayerNorm of q and k at qk_norm_eps, optional rope2d of q and k, then the core.
// q and k are copied, not mutated.  Any of qn_g/kn_g/pos_yx may be NULL (disabled).
void oracle_op_attention(const float* q, const float* k, const float* v, int heads, int64_t n,
                         int d, const float* qn_g, const float* qn_b, const float* kn_g,
                         const float* kn_b, float qk_norm_eps, const float* pos_yx, float freq,
                         int pairing, float* out, int threads) {
  threads = resolve_threads(threads);
  std::vector<float> qc(q, q + (size_t)heads * n * d), kc(k, k + (size_t)heads * n * d);
  if (qn_g) layernorm_rows(qc.data(), (int64_t)heads * n, d, qn_g, qn_b, qk_norm_eps, threads);
  if (kn_g) layernorm_rows(kc.data(), (int64_t)heads * n, d, kn_g, kn_b, qk_norm_eps, threads);
  if (pos_yx) {
    rope2d(qc.data(), heads, n, d, pos_yx, freq, pairing, threads);
    rope2d(kc.data(), heads, n, d, pos_yx, freq, pairing, threads);
  }
  attention_core(qc.data(), kc.data(), v, heads, n, d, n, nullptr, 0, out, threads);
}

// The attention sub-block of one ViT block (vit_block.rs:772-992):
//   ln1 [rows, E] -> QKV = ln1 * qkv_w + qkv_b  (qkv_w [E, 3E], columns [Q|K|V],
//   each [heads, d] head-major, vit_block.rs:39-43) -> q,k,v [heads, rows, d]
//   -> QK-norm (if qn_g) -> RoPE (if pos_yx) -> attention over segments of
//   seg_len tokens -> token-major [rows, E] -> proj_w [E, E] + proj_b (* ls1 if given).
// q_rows (optional, nq entries, ascending) restricts the output to those token rows
// (out is then [nq, E]); K and V are still formed for every row.
// Returns 0 on success, -1 on a shape error.
int oracle_attention_block(const float* ln1, int64_t rows, int E, int heads, int d,
                           const float* qkv_w, const float* qkv_b, const float* qn_g,
                           const float* qn_b, const float* kn_g, const float* kn_b,
                           float qk_norm_eps, const float* pos_yx, float rope_freq, int pairing,
                           int64_t seg_len, const float* proj_w, const float* proj_b,
                           const float* ls1, const int64_t* q_rows, int64_t nq, float* out,
                           int threads) {
  if (heads * d != E || rows <= 0 || (seg_len > 0 && rows % seg_len != 0)) return -1;
  threads = resolve_threads(threads);
  if (seg_len <= 0) seg_len = rows;
  const int64_t nrows = q_rows ? nq : rows;
  // K and V need every row; Q only the requested rows.
  std::vector<float> kv((size_t)rows * 2 * E);
  {
    // K|V columns of the fused weight: gather them into a [E, 2E] panel.
    std::vector<float> wkv((size_t)E * 2 * E), bkv(2 * (size_t)E);
    for (int i = 0; i < E; ++i)
      std::memcpy(&wkv[(size_t)i * 2 * E], qkv_w + (size_t)i * 3 * E + E, sizeof(float) * 2 * E);
    std::memcpy(bkv.data(), qkv_b + E, sizeof(float) * 2 * E);
    linear(ln1, rows, E, wkv.data(), 2 * E, bkv.data(), nullptr, kv.data(), threads);
  }
  std::vector<float> qtok((size_t)nrows * E);
  {
    std::vector<float> wq((size_t)E * E);
    for (int i = 0; i < E; ++i)
      std::memcpy(&wq[(size_t)i * E], qkv_w + (size_t)i * 3 * E, sizeof(float) * E);
    if (q_rows) {
      std::vector<float> sel((size_t)nq * E);
      for (int64_t i = 0; i < nq; ++i)
        std::memcpy(&sel[(size_t)i * E], ln1 + q_rows[i] * E, sizeof(float) * E);
      linear(sel.data(), nq, E, wq.data(), E, qkv_b, nullptr, qtok.data(), threads);
    } else {
      linear(ln1, rows, E, wq.data(), E, qkv_b, nullptr, qtok.data(), threads);
    }
  }
  // Head split: token-major -> [heads, rows, d] (vit_block.rs:817-831).
  std::vector<float> q((size_t)heads * nrows * d), k((size_t)heads * rows * d),
      v((size_t)heads * rows * d);
#pragma omp parallel for num_threads(threads) schedule(static)
  for (int64_t t = 0; t < rows; ++t)
    for (int h = 0; h < heads; ++h) {
      std::memcpy(&k[((size_t)h * rows + t) * d], &kv[(size_t)t * 2 * E + h * d], sizeof(float) * d);
      std::memcpy(&v[((size_t)h * rows + t) * d], &kv[(size_t)t * 2 * E + E + h * d],
                  sizeof(float) * d);
    }
#pragma omp parallel for num_threads(threads) schedule(static)
  for (int64_t t = 0; t < nrows; ++t)
    for (int h = 0; h < heads; ++h)
      std::memcpy(&q[((size_t)h * nrows + t) * d], &qtok[(size_t)t * E + h * d], sizeof(float) * d);
  // QK-norm then RoPE (vit_block.rs:895-948).
  if (qn_g) layernorm_rows(q.data(), (int64_t)heads * nrows, d, qn_g, qn_b, qk_norm_eps, threads);
  if (kn_g) layernorm_rows(k.data(), (int64_t)heads * rows, d, kn_g, kn_b, qk_norm_eps, threads);
  if (pos_yx) {
    std::vector<float> qpos((size_t)nrows * 2);
    for (int64_t i = 0; i < nrows; ++i) {
      const int64_t t = q_rows ? q_rows[i] : i;
      qpos[2 * i] = pos_yx[2 * t];
      qpos[2 * i + 1] = pos_yx[2 * t + 1];
    }
    rope2d(q.data(), heads, nrows, d, qpos.data(), rope_freq, pairing, threads);
    rope2d(k.data(), heads, rows, d, pos_yx, rope_freq, pairing, threads);
  }
  // Core.  With a row subset, Q holds only those rows, so the core runs against
  // the full K/V with explicit query indices.
  std::vector<float> o((size_t)heads * nrows * d);
  if (q_rows) {
    // attention_core indexes q by the absolute token; build an absolute-indexed view.
    std::vector<float> qabs((size_t)heads * rows * d, 0.f);
    for (int h = 0; h < heads; ++h)
      for (int64_t i = 0; i < nq; ++i)
        std::memcpy(&qabs[((size_t)h * rows + q_rows[i]) * d], &q[((size_t)h * nq + i) * d],
                    sizeof(float) * d);
    attention_core(qabs.data(), k.data(), v.data(), heads, rows, d, seg_len, q_rows, nq, o.data(),
                   threads);
  } else {
    attention_core(q.data(), k.data(), v.data(), heads, rows, d, seg_len, nullptr, 0, o.data(),
                   threads);
  }
  // Unpack [heads, rows, d] -> token-major (vit_block.rs:957-965), then projection.
  std::vector<float> otok((size_t)nrows * E);
#pragma omp parallel for num_threads(threads) schedule(static)
  for (int64_t t = 0; t < nrows; ++t)
    for (int h = 0; h < heads; ++h)
      std::memcpy(&otok[(size_t)t * E + h * d], &o[((size_t)h * nrows + t) * d], sizeof(float) * d);
  linear(otok.data(), nrows, E, proj_w, E, proj_b, ls1, out, threads);
  return 0;
}

// Double-precision naive attention (materialised scores) for small cases; used to
// check the online-softmax core above.
// MLP sub-block of one ViT block (vit_block.rs:1092-1129, device form :566-580):
//   out = x + (GELU(LN2(x) @ fc1_w + fc1_b) @ fc2_w + fc2_b) * ls2
// with GELU(z) = z/2 * (1 + erf(z / sqrt(2))) (the module doc, vit_block.rs:26),
// LN2 eps = ln_eps, ls2 presence-gated (null: unscaled).  Weights [in, out].
// x, out: [rows, E]; they may alias (the residual is read before it is written).
void oracle_mlp_block(const float* x, int64_t rows, int E, int hidden, const float* n2_g,
                      const float* n2_b, float ln_eps, const float* fc1_w, const float* fc1_b,
                      const float* fc2_w, const float* fc2_b, const float* ls2, float* out,
                      int threads) {
  threads = resolve_threads(threads);
  std::vector<float> ln((size_t)rows * E);
  std::memcpy(ln.data(), x, sizeof(float) * ln.size());
  layernorm_rows(ln.data(), rows, E, n2_g, n2_b, ln_eps, threads);
  std::vector<float> h((size_t)rows * hidden);
  linear(ln.data(), rows, E, fc1_w, hidden, fc1_b, nullptr, h.data(), threads);
#pragma omp parallel for num_threads(threads) schedule(static)
  for (int64_t i = 0; i < (int64_t)h.size(); ++i) {
    const float z = h[i];
    h[i] = 0.5f * z * (1.0f + std::erf(z * 0.70710678118654752f));
  }
  std::vector<float> m((size_t)rows * E);
  linear(h.data(), rows, hidden, fc2_w, E, fc2_b, ls2, m.data(), threads);
#pragma omp parallel for num_threads(threads) schedule(static)
  for (int64_t i = 0; i < (int64_t)m.size(); ++i) out[i] = x[i] + m[i];
}

void oracle_attention_naive_f64(const double* q, const double* k, const double* v, int heads,
                                int64_t n, int d, int64_t seg_len, double* out) {
  if (seg_len <= 0) seg_len = n;
  const double scale = 1.0 / std::sqrt((double)d);
  std::vector<double> s;
  for (int h = 0; h < heads; ++h)
    for (int64_t i = 0; i < n; ++i) {
      const int64_t kb = (i / seg_len) * seg_len, ke = std::min(n, kb + seg_len);
      s.assign((size_t)(ke - kb), 0.0);
      double mx = -std::numeric_limits<double>::infinity();
      for (int64_t t = kb; t < ke; ++t) {
        double acc = 0.0;
        for (int c = 0; c < d; ++c) acc += q[((size_t)h * n + i) * d + c] * k[((size_t)h * n + t) * d + c];
        s[(size_t)(t - kb)] = acc * scale;
        mx = std::max(mx, acc * scale);
      }
      double l = 0.0;
      for (auto& x : s) {
        x = std::exp(x - mx);
        l += x;
      }
      for (int c = 0; c < d; ++c) {
        double acc = 0.0;
        for (int64_t t = kb; t < ke; ++t) acc += s[(size_t)(t - kb)] * v[((size_t)h * n + t) * d + c];
        out[((size_t)h * n + i) * d + c] = acc / l;
      }
    }
}

}  // extern "C"
