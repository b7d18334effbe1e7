// K1 / K3: tcgen05 BF16 GEMMs with fused epilogues.
//
//   C[M, N] = A[M, K] * B[N, K]^T        (both operands K-major in HBM)
//
// K1 (QKV projection, vit_block.rs:803-831 + :895-948): A = LN1 output (bf16),
//   B = W_qkv^T [3E, E].  Epilogue per 64-column head chunk: + bias, then for the
//   Q and K sections per-head LayerNorm (eps 1e-5, vit_block.rs:686) and 2D RoPE,
//   cast to bf16 and store token-major [rows][E] per section (the split_qkv layout
//   transform: head h occupies columns [64h, 64h+64), one 128-B row per thread).
// K3 (output projection, vit_block.rs:969-979 -> run_linear :721-761): A = attention
//   output O (token-major bf16), B = W_proj^T [E, E].  Epilogue: + bias, * ls1 when
//   present, + residual when asked (vit_block.rs:1090), F32 store.
//
// Structure: one 128 x BN output tile per CTA, 10 warps, two CTAs per SM (the
// STAGES-deep ring is sized for that), so one CTA's epilogue overlaps the other's
// main loop.
//   warp 0      TMA producer (one elected lane), STAGES-deep smem ring
//   warp 1      TMEM allocator + single-thread UMMA issuer (M=128, N=BN, K=16 steps)
//   warps 2..9  epilogue: warp w reads TMEM lanes 32*(w%4)..+31 (tile rows), one
//               row per thread; warps 2..5 take columns [0, BN/2), warps 6..9
//               [BN/2, BN).
// Operands arrive through TMA with SWIZZLE_128B (64 bf16 = one 128-B row per
// box row), which is exactly the UMMA K-major SW128 canonical layout.
#include <math.h>

#include <algorithm>
#include <cstdlib>

#include "va_internal.h"
#include "va_ptx.cuh"

namespace va {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kGemmThreads = 320;

__device__ __forceinline__ float ln_rsqrt(float var_eps) { return 1.0f / sqrtf(var_eps); }

// LayerNorm of one 64-wide head row held in registers (torch semantics); g and b
// point at the affine parameters in shared memory.
__device__ __forceinline__ void head_layernorm(float* x, const float* g, const float* b, float eps) {
  float mean = 0.f;
#pragma unroll
  for (int i = 0; i < 64; ++i) mean += x[i];
  mean *= (1.0f / 64.0f);
  float var = 0.f;
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    const float d = x[i] - mean;
    var += d * d;
  }
  var *= (1.0f / 64.0f);
  const float inv = ln_rsqrt(var + eps);
#pragma unroll
  for (int i = 0; i < 64; ++i) x[i] = (x[i] - mean) * inv * g[i] + b[i];
}

// 2D RoPE of one 64-wide head row: channels [0,32) rotate with y, [32,64) with x.
// The table is i-major ([16][npos]): the 32 rows of a warp are consecutive tokens, so
// their positions are equal (y) or consecutive (x within a row of patches) and each
// load of one frequency touches one or two cache lines across the warp.
__device__ __forceinline__ void head_rope(float* x, int2 pos, const float2* cs, int npos, int pairing) {
#pragma unroll
  for (int axis = 0; axis < 2; ++axis) {
    const float2* col = cs + (axis == 0 ? pos.x : pos.y);
    float* seg = x + axis * 32;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float2 c = __ldg(col + i * npos);
      if (pairing == 0) {
        const float a = seg[i], bb = seg[i + 16];
        seg[i] = a * c.x - bb * c.y;
        seg[i + 16] = bb * c.x + a * c.y;
      } else {
        const float a = seg[2 * i], bb = seg[2 * i + 1];
        seg[2 * i] = a * c.x - bb * c.y;
        seg[2 * i + 1] = bb * c.x + a * c.y;
      }
    }
  }
}

// erf(x) by Abramowitz & Stegun, Handbook of Mathematical Functions, formula 7.1.26:
//   erf(x) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-x^2),  t = 1 / (1 + p x),
// x >= 0, odd extension for x < 0, |error| <= 1.5e-7 (about 5e-7 evaluated in F32;
// GELU's absolute error then stays below 4e-7, far under the bf16 rounding of the
// fc1 output it feeds).  One reciprocal and one exp2 on MUFU plus a short FMA chain.
__device__ __forceinline__ float erf_as7126(float x) {
  const float ax = fabsf(x);
  float t;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(fmaf(0.3275911f, ax, 1.0f)));
  float poly = fmaf(1.061405429f, t, -1.453152027f);
  poly = fmaf(poly, t, 1.421413741f);
  poly = fmaf(poly, t, -0.284496736f);
  poly = fmaf(poly, t, 0.254829592f);
  poly *= t;
  float e;  // exp(-x^2) = 2^(-x^2 log2 e)
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-ax * ax * 1.4426950408889634f));
  return copysignf(fmaf(-poly, e, 1.0f), x);
}

// bf16 (or f16) of 8 consecutive values as one 16-byte chunk.
__device__ __forceinline__ uint4 pack8(const float* x, bool f16) {
  uint4 u;
  if (f16) {
    u.x = f16x2_from_f32(x[0], x[1]);
    u.y = f16x2_from_f32(x[2], x[3]);
    u.z = f16x2_from_f32(x[4], x[5]);
    u.w = f16x2_from_f32(x[6], x[7]);
  } else {
    u.x = pack_bf16x2(x[0], x[1]);
    u.y = pack_bf16x2(x[2], x[3]);
    u.z = pack_bf16x2(x[4], x[5]);
    u.w = pack_bf16x2(x[6], x[7]);
  }
  return u;
}

// Epilogue contract (warps 2..9 of the GEMM CTA, 256 threads):
//   stage(cbuf, n0, t)  thread t < 256 copies its share of the tile's per-column
//                       constants into shared memory, before the accumulator is ready;
//   run(...)            thread (quad, half) turns TMEM row r, columns of its half, into
//                       output values and writes them as 16 KB SWIZZLE_128B tiles of
//                       128 rows x 128 B into the (by then idle) operand ring;
//   store(...)          one thread of each half sends that half's tiles out by TMA.
// Rows past M are computed from the zero-filled operands and clipped by the store.
constexpr uint32_t kOutTileBytes = 16384;

struct QkvEpilogue {
  QkvEpilogueArgs a;
  CUtensorMap map_out[3];  // Q, K, V: [rows][E] 2-byte, box 64 x 128

  __device__ __forceinline__ uint32_t prefetch_bytes(int = 1) const { return 0; }
  __device__ __forceinline__ void prefetch(int, int, int, uint32_t, uint32_t, int = 0, int = 1) const {}

  // cbuf: [0, 256) bias of the tile's columns, [256, 320) gamma, [320, 384) beta of
  // the section's QK-norm (1 and 0 when the section has none).
  __device__ __forceinline__ void stage(float* cbuf, int n0, int t) const {
    const int section = n0 / a.embed;
    cbuf[t] = a.bias[n0 + t];
    if (t < 64) {
      const float* g = section == 0 ? a.q_g : a.k_g;
      const float* b = section == 0 ? a.q_b : a.k_b;
      const bool norm = section < 2 && g != nullptr;
      cbuf[256 + t] = norm ? g[t] : 1.0f;
      cbuf[320 + t] = norm ? b[t] : 0.0f;
    }
  }

  template <int BN>
  __device__ __forceinline__ void run(uint32_t tmem_row, int r, int m0, int n0, int half,
                                      const float* cbuf, uint32_t out_smem, bool valid, int cp = 0,
                                      int ncp = 1) const {
    static_assert(BN == 256, "QKV tiles are 4 heads wide");
    const int section = n0 / a.embed;  // 0 = Q, 1 = K, 2 = V
    const bool norm = section < 2 && (section == 0 ? a.q_g : a.k_g) != nullptr;
    const bool rope = section < 2 && a.pos != nullptr;
    const bool f16 = section == 2 && a.v_f16;
    const int2 pos = (rope && valid) ? a.pos[m0 + r] : make_int2(0, 0);
#pragma unroll 1
    for (int j = 0; j < 2; ++j) {
      const int hh = half * 2 + j;
      float x[64];
      tmem_ld32(tmem_row + hh * 64, x);
      tmem_ld32(tmem_row + hh * 64 + 32, x + 32);
      if (valid) {
        const float4* bias = reinterpret_cast<const float4*>(cbuf + hh * 64);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float4 v = bias[i];
          x[4 * i] += v.x;
          x[4 * i + 1] += v.y;
          x[4 * i + 2] += v.z;
          x[4 * i + 3] += v.w;
        }
        if (norm) head_layernorm(x, cbuf + 256, cbuf + 320, a.qk_eps);
        if (rope) head_rope(x, pos, a.rope_cs, a.rope_npos, a.rope_pairing);
      }
      const uint32_t tile = out_smem + hh * kOutTileBytes;
#pragma unroll
      for (int c = 0; c < 8; ++c) st_shared_v4(tile + sw128_offset(r, c), pack8(x + 8 * c, f16));
    }
  }

  // Direct K'/V exchange: the 128 threads of `half` copy this half's two output
  // tiles (K or V section) row-major from shared memory into every peer's window,
  // rows < M only (the rows past M belong to the next rank's slice there).  Each
  // warp instruction covers 4 whole 128-byte rows.  Fenced at system scope.
  __device__ __forceinline__ void peer_copy(int half, int t, int m0, int M, int n0,
                                            uint32_t out_smem) const {
    const int section = n0 / a.embed;
    if (a.npeer == 0 || section == 0) return;
    const int h0 = (n0 - section * a.embed) / 64;
    const int chunk = t & 7;
    for (int j = 0; j < 2; ++j) {
      const int hh = half * 2 + j;
      const uint32_t tile = out_smem + hh * kOutTileBytes;
#pragma unroll 2
      for (int i = 0; i < 8; ++i) {
        const int r = (t >> 3) + 16 * i;
        if (m0 + r >= M) break;
        const uint4 v = ld_shared_v4(tile + sw128_offset(r, chunk));
        const size_t off = static_cast<size_t>(m0 + r) * a.embed + (h0 + hh) * 64 + chunk * 8;
        for (int p = 0; p < a.npeer; ++p) {
          __nv_bfloat16* dst = (section == 1 ? a.peer_k[p] : a.peer_v[p]) + off;
          *reinterpret_cast<uint4*>(dst) = v;
        }
      }
    }
    __threadfence_system();
  }

  __device__ __forceinline__ void store(int half, int m0, int n0, uint32_t out_smem, int cp = 0,
                                        int ncp = 1) const {
    const int section = n0 / a.embed;
    const int h0 = (n0 - section * a.embed) / 64;
    for (int j = 0; j < 2; ++j) {
      const int hh = half * 2 + j;
      tma_store_2d(&map_out[section], out_smem + hh * kOutTileBytes, (h0 + hh) * 64, m0);
    }
    bulk_commit_group();
  }
};

// MLP fc1 (vit_block.rs:1106-1115 / device :578): + bias, GELU with the exact erf
// form z/2 * (1 + erf(z/sqrt 2)) (module doc, vit_block.rs:26), bf16 hidden out.
struct Fc1Epilogue {
  Fc1EpilogueArgs a;
  CUtensorMap map_out;  // bf16 [rows][hidden], box 64 x 128

  __device__ __forceinline__ uint32_t prefetch_bytes(int = 1) const { return 0; }
  __device__ __forceinline__ void prefetch(int, int, int, uint32_t, uint32_t, int = 0, int = 1) const {}

  __device__ __forceinline__ void stage(float* cbuf, int n0, int t) const { cbuf[t] = a.bias[n0 + t]; }

  template <int BN>
  __device__ __forceinline__ void run(uint32_t tmem_row, int r, int m0, int n0, int half,
                                      const float* cbuf, uint32_t out_smem, bool valid, int cp = 0,
                                      int ncp = 1) const {
    static_assert(BN == 256, "fc1 tiles are 256 columns wide");
#pragma unroll 1
    for (int j = 0; j < 2; ++j) {
      const int hh = half * 2 + j;  // 64-column block
      float x[64];
      tmem_ld32(tmem_row + hh * 64, x);
      tmem_ld32(tmem_row + hh * 64 + 32, x + 32);
      if (valid) {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float z = x[i] + cbuf[hh * 64 + i];
          x[i] = 0.5f * z * (1.0f + erf_as7126(z * 0.70710678118654752f));
        }
      }
      const uint32_t tile = out_smem + hh * kOutTileBytes;
#pragma unroll
      for (int c = 0; c < 8; ++c) st_shared_v4(tile + sw128_offset(r, c), pack8(x + 8 * c, false));
    }
  }

  __device__ __forceinline__ void peer_copy(int, int, int, int, int, uint32_t) const {}

  __device__ __forceinline__ void store(int half, int m0, int n0, uint32_t out_smem, int cp = 0,
                                        int ncp = 1) const {
    for (int j = 0; j < 2; ++j) {
      const int hh = half * 2 + j;
      tma_store_2d(&map_out, out_smem + hh * kOutTileBytes, n0 + hh * 64, m0);
    }
    bulk_commit_group();
  }
};

struct ProjEpilogue {
  ProjEpilogueArgs a;
  CUtensorMap map_out;  // F32 [rows][embed], box 32 x 128
  CUtensorMap map_res;  // the residual, same boxes (persistent kernel: prefetched by TMA)
  int res_staged = 0;   // 1: the residual tile is already in the staging tiles when run() starts

  // Column passes: with ncp = 2 a pass handles one of each half's two 32-column
  // chunks and the staging area holds two tiles (slot = half); with ncp = 1 all four
  // chunks at once (slot = chunk).
  // Bytes one half's store thread prefetches into its staging tiles per pass.
  __device__ __forceinline__ uint32_t prefetch_bytes(int ncp = 1) const {
    return res_staged ? (2 / ncp) * kOutTileBytes : 0;
  }
  __device__ __forceinline__ void prefetch(int half, int m0, int n0, uint32_t out_smem, uint32_t bar,
                                           int cp = 0, int ncp = 1) const {
    for (int j = 0; j < 2; ++j) {
      if (ncp == 2 && j != cp) continue;
      const int chunk = half * 2 + j, slot = ncp == 1 ? chunk : half;
      tma_load_2d(out_smem + slot * kOutTileBytes, &map_res, bar, n0 + chunk * 32, m0);
    }
  }

  // cbuf: [0, 128) bias (0 when absent), [128, 256) ls1 (1 when absent).
  __device__ __forceinline__ void stage(float* cbuf, int n0, int t) const {
    if (t < 128)
      cbuf[t] = a.bias ? a.bias[n0 + t] : 0.0f;
    else
      cbuf[t] = a.ls1 ? a.ls1[n0 + t - 128] : 1.0f;
  }

  template <int BN>
  __device__ __forceinline__ void run(uint32_t tmem_row, int r, int m0, int n0, int half,
                                      const float* cbuf, uint32_t out_smem, bool valid, int cp = 0,
                                      int ncp = 1) const {
    static_assert(BN == 128, "projection tiles are 128 columns wide");
#pragma unroll 1
    for (int j = 0; j < 2; ++j) {
      if (ncp == 2 && j != cp) continue;
      const int chunk = half * 2 + j;  // 32 columns
      const int slot = ncp == 1 ? chunk : half;
      float x[32];
      tmem_ld32(tmem_row + chunk * 32, x);
      if (valid) {
        const float* bias = cbuf + chunk * 32;
        const float* ls1 = cbuf + 128 + chunk * 32;
#pragma unroll
        for (int i = 0; i < 32; ++i) x[i] = (x[i] + bias[i]) * ls1[i];
        if (a.residual && res_staged) {
          const uint32_t tile = out_smem + slot * kOutTileBytes;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 v = ld_shared_v4(tile + sw128_offset(r, c));
            x[4 * c] += __uint_as_float(v.x);
            x[4 * c + 1] += __uint_as_float(v.y);
            x[4 * c + 2] += __uint_as_float(v.z);
            x[4 * c + 3] += __uint_as_float(v.w);
          }
        } else if (a.residual) {
          const float4* res = reinterpret_cast<const float4*>(
              a.residual + static_cast<size_t>(m0 + r) * a.embed + n0 + chunk * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 v = res[i];
            x[4 * i] += v.x;
            x[4 * i + 1] += v.y;
            x[4 * i + 2] += v.z;
            x[4 * i + 3] += v.w;
          }
        }
      }
      const uint32_t tile = out_smem + slot * kOutTileBytes;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        st_shared_v4(tile + sw128_offset(r, c),
                     make_uint4(__float_as_uint(x[4 * c]), __float_as_uint(x[4 * c + 1]),
                                __float_as_uint(x[4 * c + 2]), __float_as_uint(x[4 * c + 3])));
    }
  }

  __device__ __forceinline__ void peer_copy(int, int, int, int, int, uint32_t) const {}

  __device__ __forceinline__ void store(int half, int m0, int n0, uint32_t out_smem, int cp = 0,
                                        int ncp = 1) const {
    for (int j = 0; j < 2; ++j) {
      if (ncp == 2 && j != cp) continue;
      const int chunk = half * 2 + j, slot = ncp == 1 ? chunk : half;
      tma_store_2d(&map_out, out_smem + slot * kOutTileBytes, n0 + chunk * 32, m0);
    }
    bulk_commit_group();
  }
};

// Patch projection (patch_embed.rs:53-133 + pos_embed.rs:254-300): + bias + the
// patch's interpolated position.  A tile whose 128 rows lie in one view is staged
// as SWIZZLE_128B F32 tiles and sent by TMA through a 3-D map (columns, patch,
// view) over the token rows after each view's specials; a tile that crosses a
// view boundary (a box cannot follow the jump over the next view's special rows)
// writes its rows directly.
struct PatchEpilogue {
  PatchEpilogueArgs a;
  CUtensorMap map_out;  // F32 (E, n_patches, views), strides (E, n_tok*E) floats, box 32 x 128 x 1

  __device__ __forceinline__ uint32_t prefetch_bytes(int = 1) const { return 0; }
  __device__ __forceinline__ void prefetch(int, int, int, uint32_t, uint32_t, int = 0, int = 1) const {}

  __device__ __forceinline__ bool one_view(int m0) const {
    const int last = min(m0 + kBM - 1, a.rows - 1);
    return m0 / a.n_patches == last / a.n_patches;
  }

  __device__ __forceinline__ void stage(float* cbuf, int n0, int t) const {
    if (t < 128) cbuf[t] = a.bias[n0 + t];
  }

  template <int BN>
  __device__ __forceinline__ void run(uint32_t tmem_row, int r, int m0, int n0, int half,
                                      const float* cbuf, uint32_t out_smem, bool valid, int cp = 0,
                                      int ncp = 1) const {
    static_assert(BN == 128, "patch tiles are 128 columns wide");
    const int m = m0 + r;
    const int view = m / a.n_patches, p = m - view * a.n_patches;
    const bool staged = one_view(m0);
#pragma unroll 1
    for (int j = 0; j < 2; ++j) {
      if (ncp == 2 && j != cp) continue;
      const int chunk = half * 2 + j;  // 32 columns
      const int slot = ncp == 1 ? chunk : half;
      float x[32];
      tmem_ld32(tmem_row + chunk * 32, x);  // warp-collective: every lane loads
      const int col = n0 + chunk * 32;
      if (valid) {
        const float4* pos = reinterpret_cast<const float4*>(a.pos + static_cast<size_t>(1 + p) * a.embed + col);
        const float* bias = cbuf + chunk * 32;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 q = __ldg(pos + i);
          x[4 * i] = x[4 * i] + bias[4 * i] + q.x;
          x[4 * i + 1] = x[4 * i + 1] + bias[4 * i + 1] + q.y;
          x[4 * i + 2] = x[4 * i + 2] + bias[4 * i + 2] + q.z;
          x[4 * i + 3] = x[4 * i + 3] + bias[4 * i + 3] + q.w;
        }
      }
      if (staged) {
        // Rows past the last patch are clipped by the store; their values are unused.
        const uint32_t tile = out_smem + slot * kOutTileBytes;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          st_shared_v4(tile + sw128_offset(r, c),
                       make_uint4(__float_as_uint(x[4 * c]), __float_as_uint(x[4 * c + 1]),
                                  __float_as_uint(x[4 * c + 2]), __float_as_uint(x[4 * c + 3])));
      } else if (valid) {
        float4* out = reinterpret_cast<float4*>(
            a.out + (static_cast<size_t>(view) * a.n_tok + a.n_special + p) * a.embed + col);
#pragma unroll
        for (int i = 0; i < 8; ++i) out[i] = make_float4(x[4 * i], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]);
      }
    }
  }

  __device__ __forceinline__ void peer_copy(int, int, int, int, int, uint32_t) const {}

  __device__ __forceinline__ void store(int half, int m0, int n0, uint32_t out_smem, int cp = 0,
                                        int ncp = 1) const {
    if (!one_view(m0)) return;
    const int view = m0 / a.n_patches, p0 = m0 - view * a.n_patches;
    for (int j = 0; j < 2; ++j) {
      if (ncp == 2 && j != cp) continue;
      const int chunk = half * 2 + j, slot = ncp == 1 ? chunk : half;
      tma_store_3d(&map_out, out_smem + slot * kOutTileBytes, n0 + chunk * 32, p0, view);
    }
    bulk_commit_group();
  }
};

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr uint32_t kABytes = kBM * kBK * 2;
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kBarOffset = STAGES * kStageBytes;
  static constexpr uint32_t kConstOffset = kBarOffset + 256;  // after barriers + tmem slot + flags
  static constexpr uint32_t kBytes = kConstOffset + 2048;     // per-column epilogue constants
  // The epilogue's output tiles reuse the operand ring once the accumulator is final.
  static_assert(4 * kOutTileBytes <= STAGES * kStageBytes, "ring too small for the output tiles");
  static constexpr uint32_t kLaunchBytes = kBytes + 1024;  // slack for 1024-B alignment
};

// Waits (bounded, ignoring the abort flag) so that nothing asynchronous still
// targets this CTA's shared memory or TMEM when it tears down after an abort.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) break;
  }
}

template <int BN, int STAGES, class Epi>
__global__ void __launch_bounds__(kGemmThreads, 2)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap map_a,
                     const __grid_constant__ CUtensorMap map_b, int M, int K,
                     const __grid_constant__ Epi epi, int* err) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - raw_u32);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * kBM;
  const int n0 = blockIdx.x * BN;
  const int num_kb = K / kBK;

  const uint32_t bar0 = base_u32 + L::kBarOffset;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  const uint32_t accum_bar = bar0 + 8u * (2 * STAGES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kBarOffset + 8 * (2 * STAGES + 1));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* issued = reinterpret_cast<volatile int*>(tmem_slot + 2);
  volatile int* consumed = reinterpret_cast<volatile int*>(tmem_slot + 3);
  volatile int* accum_seen = reinterpret_cast<volatile int*>(tmem_slot + 4);
  auto sA = [&](int s) { return base_u32 + s * L::kStageBytes; };
  auto sB = [&](int s) { return base_u32 + s * L::kStageBytes + L::kABytes; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(accum_bar, 1);
    *abort_flag = 0;
    *issued = 0;
    *consumed = 0;
    *accum_seen = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (!mbar_wait(empty_bar(s), ph ^ 1, abort_flag, err, kDevTimeoutProducer)) break;
        mbar_arrive_expect_tx(full_bar(s), L::kStageBytes);
        tma_load_2d(sA(s), &map_a, full_bar(s), kb * kBK, m0);
        tma_load_2d(sB(s), &map_b, full_bar(s), kb * kBK, n0);
        *issued = kb + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kBM, BN, false, false);
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (!mbar_wait(full_bar(s), ph, abort_flag, err, kDevTimeoutMma)) break;
        *consumed = kb + 1;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          const uint64_t ad = sdesc_sw128(sA(s) + k * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(sB(s) + k * 32, 16, 1024);
          umma_ss(tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
        }
        tc_commit(empty_bar(s));
      }
      tc_commit(accum_bar);
    }
  } else {
    // Epilogue warps 2..9.  Every one of them reaches both named barriers: the
    // accumulator wait is bounded and nothing else waits in between.
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // warps 2..5 -> 0, 6..9 -> 1
    const int row = quad * 32 + lane;
    float* cbuf = reinterpret_cast<float*>(smem + L::kConstOffset);
    epi.stage(cbuf, n0, threadIdx.x - 64);
    named_bar_sync(1, 256);
    bool ok = mbar_wait(accum_bar, 0, abort_flag, err, kDevTimeoutConsumer);
    ok = __all_sync(0xffffffffu, ok);  // reconverge: tcgen05.ld is warp-collective
    if (ok) {
      if (lane == 0) *accum_seen = 1;
      tc_fence_after();
      epi.template run<BN>(tmem + (static_cast<uint32_t>(quad * 32) << 16), row, m0, n0, half, cbuf,
                           base_u32, (m0 + row) < M);
    }
    fence_proxy_async_smem();  // the tiles written above are read by the TMA store
    named_bar_sync(2 + half, 128);
    if (ok && ((warp - 2) & 3) == 0 && lane == 0) {
      epi.store(half, m0, n0, base_u32);
      bulk_wait_all();  // the ring may not be released while the store reads it
    }
    if (ok) epi.peer_copy(half, threadIdx.x - 64 - 128 * half, m0, M, n0, base_u32);
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) {
    // Drain TMA copies that were issued but never consumed, then the UMMAs.
    for (int kb = *consumed; kb < *issued; ++kb) drain_wait(full_bar(kb % STAGES), (kb / STAGES) & 1);
    if (!*accum_seen) drain_wait(accum_bar, 0);
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

template <int BN, int STAGES, class Epi>
cudaError_t launch_gemm(const __nv_bfloat16* a, const __nv_bfloat16* b, int M, int N, int K,
                        const Epi& epi, int* err, cudaStream_t st) {
  if (M <= 0 || N % BN != 0 || K % kBK != 0) return cudaErrorInvalidValue;
  CUtensorMap map_a, map_b;
  if (!encode_tma_2d_bf16(&map_a, a, K, M, kBK, kBM)) return cudaErrorInvalidValue;
  if (!encode_tma_2d_bf16(&map_b, b, K, N, kBK, BN)) return cudaErrorInvalidValue;
  using L = GemmSmem<BN, STAGES>;
  auto kern = gemm_bf16_kernel<BN, STAGES, Epi>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       L::kLaunchBytes);
  if (e != cudaSuccess) return e;
  dim3 grid(N / BN, (M + kBM - 1) / kBM);
  kern<<<grid, kGemmThreads, L::kLaunchBytes, st>>>(map_a, map_b, M, K, epi, err);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Persistent form: one CTA per SM walks tiles blockIdx.x, +gridDim.x, ...
//   warp 0      TMA producer over all tiles' K slabs (STAGES-deep ring)
//   warp 1      TMEM owner + UMMA issuer; tile i accumulates into TMEM buffer i&1
//   warps 2..9  epilogue of tile i from buffer i&1 while tile i+1 accumulates
//               into the other; output tiles staged in their own 64 KB region
// so neither the operand loads nor the epilogue wait for each other across tiles.
// A tile is MT x 128 rows by BN columns: MT = 2 gives each loaded B slab twice the
// UMMA work (two M=128 accumulators side by side in TMEM), which halves the B
// traffic per FLOP of the narrow (N = E) projections; the epilogue then runs one
// pass per 128-row half.
// ---------------------------------------------------------------------------
template <int BN, int MT, int STAGES, int CP>
struct PersistentSmem {
  static constexpr uint32_t kABytes = MT * kBM * kBK * 2;
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kStagingOffset = STAGES * kStageBytes;
  // CP column passes per 128-row pass: the staging area holds 4 / CP output tiles.
  static constexpr uint32_t kBarOffset = kStagingOffset + (4 / CP) * kOutTileBytes;
  // full[S], empty[S], tmem_full[2], tmem_empty[2], final, prefetch[2]; then the TMEM
  // slot and flags
  static constexpr uint32_t kNumBars = 2 * STAGES + 7;
  static constexpr uint32_t kSlotOffset = kBarOffset + 8 * kNumBars;
  static constexpr uint32_t kConstOffset = kBarOffset + 256;
  static constexpr uint32_t kBytes = kConstOffset + 1536;  // 384 per-column constants
  static constexpr uint32_t kLaunchBytes = kBytes + 1024;
  static_assert(kSlotOffset + 32 <= kConstOffset, "barrier region too small");
  static_assert(kLaunchBytes <= 227 * 1024, "shared memory budget");
  static_assert(kStageBytes % 1024 == 0, "SW128 tiles need 1024-byte alignment");
  static_assert(2 * MT * BN <= 512, "two accumulator buffers must fit in TMEM");
};

template <int BN, int MT, int STAGES, int CP, class Epi>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_persistent(const __grid_constant__ CUtensorMap map_a,
                         const __grid_constant__ CUtensorMap map_b, int M, int K, int n_tiles_n,
                         int num_tiles, const __grid_constant__ Epi epi, int* err) {
  using L = PersistentSmem<BN, MT, STAGES, CP>;
  constexpr int kTileM = MT * kBM;
  constexpr uint32_t kTmemCols = 2 * MT * BN;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - raw_u32);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_kb = K / kBK;

  const uint32_t bar0 = base_u32 + L::kBarOffset;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int b) { return bar0 + 8u * (2 * STAGES + b); };
  auto tempty_bar = [&](int b) { return bar0 + 8u * (2 * STAGES + 2 + b); };
  const uint32_t final_bar = bar0 + 8u * (2 * STAGES + 4);
  auto pre_bar = [&](int h) { return bar0 + 8u * (2 * STAGES + 5 + h); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kSlotOffset);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* issued = reinterpret_cast<volatile int*>(tmem_slot + 2);
  volatile int* consumed = reinterpret_cast<volatile int*>(tmem_slot + 3);
  volatile int* mma_started = reinterpret_cast<volatile int*>(tmem_slot + 4);
  auto sA = [&](int s) { return base_u32 + s * L::kStageBytes; };
  auto sB = [&](int s) { return base_u32 + s * L::kStageBytes + L::kABytes; };
  const uint32_t staging = base_u32 + L::kStagingOffset;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), 256);
    }
    mbar_init(final_bar, 1);
    mbar_init(pre_bar(0), 1);
    mbar_init(pre_bar(1), 1);
    *abort_flag = 0;
    *issued = 0;
    *consumed = 0;
    *mma_started = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        const int m0 = (tile / n_tiles_n) * kTileM, n0 = (tile % n_tiles_n) * BN;
        for (int kb = 0; kb < num_kb; ++kb, ++g) {
          const int s = g % STAGES;
          const uint32_t ph = (g / STAGES) & 1;
          if (!(ok = mbar_wait(empty_bar(s), ph ^ 1, abort_flag, err, kDevTimeoutProducer))) break;
          mbar_arrive_expect_tx(full_bar(s), L::kStageBytes);
          tma_load_2d(sA(s), &map_a, full_bar(s), kb * kBK, m0);
          tma_load_2d(sB(s), &map_b, full_bar(s), kb * kBK, n0);
          *issued = g + 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kBM, BN, false, false);
      *mma_started = 1;
      int g = 0, i = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++i) {
        const int b = i & 1;
        // The epilogue has drained this buffer (tile i-2).
        if (!(ok = mbar_wait(tempty_bar(b), ((i >> 1) & 1) ^ 1, abort_flag, err, kDevTimeoutMma))) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * MT * BN;
        for (int kb = 0; kb < num_kb; ++kb, ++g) {
          const int s = g % STAGES;
          const uint32_t ph = (g / STAGES) & 1;
          if (!(ok = mbar_wait(full_bar(s), ph, abort_flag, err, kDevTimeoutMma))) break;
          *consumed = g + 1;
          tc_fence_after();
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) {
              const uint64_t ad = sdesc_sw128(sA(s) + mt * kBM * 128 + k * 32, 16, 1024);
              const uint64_t bd = sdesc_sw128(sB(s) + k * 32, 16, 1024);
              umma_ss(acc + mt * BN, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
            }
          tc_commit(empty_bar(s));
        }
        if (ok) tc_commit(tfull_bar(b));
      }
      // Always committed: marks the moment every UMMA of this CTA has finished.
      tc_commit(final_bar);
    }
  } else {
    // Epilogue warps 2..9.  The tile loop has the same trip count for all 256
    // threads and never exits early, so every named barrier completes; after an
    // abort the work is skipped.
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // warps 2..5 -> 0, 6..9 -> 1
    const int row = quad * 32 + lane;
    const int t = threadIdx.x - 64;
    const bool store_thread = ((warp - 2) & 3) == 0 && lane == 0;
    float* cbuf = reinterpret_cast<float*>(smem + L::kConstOffset);
    const uint32_t pre_bytes = epi.prefetch_bytes(CP);
    int i = 0, pre_uses = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++i) {
      const int b = i & 1;
      const int n0 = (tile % n_tiles_n) * BN;
      bool ok = true;
      for (int sub = 0; sub < MT * CP; ++sub) {
        const int pass = sub / CP, cp = sub % CP;  // 128-row pass, column pass
        const int m0 = (tile / n_tiles_n) * kTileM + pass * kBM;
        // A second half that starts past the last row has nothing to load or store.
        const bool rows_here = m0 < M;
        const bool pre = pre_bytes != 0 && rows_here;
        // The previous pass's stores have read the staging tiles, and every thread
        // is done with its constants and its peer copies.
        if (store_thread) bulk_wait_all_read();
        named_bar_sync(1, 256);
        // Operands of the epilogue that do not depend on the accumulator (the
        // residual tile) start loading into this half's staging tiles now.
        if (pre && store_thread) {
          mbar_arrive_expect_tx(pre_bar(half), pre_bytes);
          epi.prefetch(half, m0, n0, staging, pre_bar(half), cp, CP);
        }
        if (sub == 0) epi.stage(cbuf, n0, t);
        named_bar_sync(1, 256);
        if (sub == 0) {
          ok = mbar_wait(tfull_bar(b), (i >> 1) & 1, abort_flag, err, kDevTimeoutConsumer);
          ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective
        }
        // Waited for even after an abort: the copy must land before the CTA exits.
        if (pre) drain_wait(pre_bar(half), (pre_uses++) & 1);
        if (ok) {
          tc_fence_after();
          epi.template run<BN>(tmem + b * MT * BN + pass * BN + (static_cast<uint32_t>(quad * 32) << 16), row,
                               m0, n0, half, cbuf, staging, (m0 + row) < M, cp, CP);
          if (sub == MT * CP - 1) {
            tc_fence_before();
            mbar_arrive(tempty_bar(b));
          }
        }
        fence_proxy_async_smem();  // the staged tiles are read by the TMA store
        named_bar_sync(2 + half, 128);
        if (ok && rows_here && store_thread) epi.store(half, m0, n0, staging, cp, CP);
        if (ok && rows_here) epi.peer_copy(half, t - 128 * half, m0, M, n0, staging);
      }
    }
    if (store_thread) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (*abort_flag)
      for (int g = *consumed; g < *issued; ++g) drain_wait(full_bar(g % STAGES), (g / STAGES) & 1);
    if (*mma_started) drain_wait(final_bar, 0);
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

int device_sms() {
  static int sms = [] {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
  }();
  return sms;
}

template <int BN, int MT, int STAGES, int CP, class Epi>
cudaError_t launch_gemm_persistent(const __nv_bfloat16* a, const __nv_bfloat16* b, int M, int N, int K,
                                   const Epi& epi, int* err, cudaStream_t st) {
  if (M <= 0 || N % BN != 0 || K % kBK != 0 || K <= 0) return cudaErrorInvalidValue;
  CUtensorMap map_a, map_b;
  if (!encode_tma_2d_bf16(&map_a, a, K, M, kBK, MT * kBM)) return cudaErrorInvalidValue;
  if (!encode_tma_2d_bf16(&map_b, b, K, N, kBK, BN)) return cudaErrorInvalidValue;
  using L = PersistentSmem<BN, MT, STAGES, CP>;
  auto kern = gemm_bf16_persistent<BN, MT, STAGES, CP, Epi>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       L::kLaunchBytes);
  if (e != cudaSuccess) return e;
  const int n_tiles_n = N / BN;
  const int num_tiles = n_tiles_n * ((M + MT * kBM - 1) / (MT * kBM));
  const int grid = std::min(num_tiles, device_sms());
  kern<<<grid, kGemmThreads, L::kLaunchBytes, st>>>(map_a, map_b, M, K, n_tiles_n, num_tiles, epi, err);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Wide projection tile (K3 and fc2 when the call has few tiles): one 256 x 256
// output tile per CTA, one launch wave.  A narrow output (N = E) cut into 256 x 128
// tiles re-reads every A row block N/128 times and leaves 1.66 waves at the DA3
// window's row count; a 256 x 256 tile reads A N/256 times and B M/256 times (a
// third less operand traffic per FLOP than 256 x 128), the tiles of a window fit in
// one wave, and with one tile per CTA the operand ring is free for the epilogue once
// the accumulator is final, so all of a 128-row pass is staged at once.
//   warp 0      TMA producer: 3 stages of A [256 x 64] + B [256 x 64] (64 KB each)
//   warp 1      TMEM (512 columns: two M=128 accumulators of N=256) + UMMA issuer
//   warps 2..9  epilogue: two 128-row passes; warp w reads TMEM lanes 32*(w%4)..,
//               warps 2..5 columns [0, 128), warps 6..9 [128, 256), four 32-column
//               SWIZZLE_128B F32 tiles each, sent by TMA.  With the residual in
//               place (out == residual) the tiles go out as TMA add-reductions:
//               out = residual + (acc + bias) * scale, one F32 add per element at
//               L2, the same single rounding as adding in registers.
// ---------------------------------------------------------------------------
struct WideSmem {
  static constexpr int kStages = 3;
  static constexpr uint32_t kABytes = 2 * kBM * kBK * 2;   // 256 rows x 64 bf16
  static constexpr uint32_t kStageBytes = kABytes + 256 * kBK * 2;
  static constexpr uint32_t kBarOffset = kStages * kStageBytes;
  // full[3], empty[3], tfull; then the TMEM slot and flags
  static constexpr uint32_t kNumBars = 2 * kStages + 1;
  static constexpr uint32_t kSlotOffset = kBarOffset + 8 * kNumBars;
  static constexpr uint32_t kConstOffset = kBarOffset + 128;
  static constexpr uint32_t kBytes = kConstOffset + 512 * 4;  // bias[256], scale[256]
  static constexpr uint32_t kLaunchBytes = kBytes + 1024;
  static_assert(kSlotOffset + 32 <= kConstOffset, "barrier region too small");
  static_assert(8 * kOutTileBytes <= kBarOffset, "a 128-row pass is staged in the operand ring");
  static_assert(kLaunchBytes <= 227 * 1024, "shared memory budget");
};

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_wide_proj(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                        const __grid_constant__ CUtensorMap map_out, ProjEpilogueArgs args, int M, int K,
                        int n_tiles_n, int reduce, int* err) {
  using L = WideSmem;
  constexpr uint32_t kTmemCols = 512;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - raw_u32);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_kb = K / kBK;
  const int m0 = (blockIdx.x / n_tiles_n) * 2 * kBM, n0 = (blockIdx.x % n_tiles_n) * 256;

  const uint32_t bar0 = base_u32 + L::kBarOffset;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (L::kStages + s); };
  const uint32_t tfull_bar = bar0 + 8u * (2 * L::kStages);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kSlotOffset);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* issued = reinterpret_cast<volatile int*>(tmem_slot + 2);
  volatile int* consumed = reinterpret_cast<volatile int*>(tmem_slot + 3);
  volatile int* mma_started = reinterpret_cast<volatile int*>(tmem_slot + 4);
  auto sA = [&](int s) { return base_u32 + s * L::kStageBytes; };
  auto sB = [&](int s) { return base_u32 + s * L::kStageBytes + L::kABytes; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < L::kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(tfull_bar, 1);
    *abort_flag = 0;
    *issued = 0;
    *consumed = 0;
    *mma_started = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    tma_prefetch_desc(&map_out);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % L::kStages;
        if (!mbar_wait(empty_bar(s), ((kb / L::kStages) & 1) ^ 1, abort_flag, err, kDevTimeoutProducer)) break;
        mbar_arrive_expect_tx(full_bar(s), L::kStageBytes);
        tma_load_2d(sA(s), &map_a, full_bar(s), kb * kBK, m0);
        tma_load_2d(sB(s), &map_b, full_bar(s), kb * kBK, n0);
        *issued = kb + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kBM, 256, false, false);
      *mma_started = 1;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % L::kStages;
        if (!mbar_wait(full_bar(s), (kb / L::kStages) & 1, abort_flag, err, kDevTimeoutMma)) break;
        *consumed = kb + 1;
        tc_fence_after();
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = sdesc_sw128(sA(s) + mt * kBM * 128 + k * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(sB(s) + k * 32, 16, 1024);
            umma_ss(tmem + mt * 256, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
        tc_commit(empty_bar(s));
      }
      // Always committed, also after an abort: it marks the moment every UMMA of
      // this CTA has finished (the epilogue and the teardown wait for it).
      tc_commit(tfull_bar);
    }
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // warps 2..5 -> 0, 6..9 -> 1
    const int row = quad * 32 + lane;
    const int t = threadIdx.x - 64;
    const bool store_thread = ((warp - 2) & 3) == 0 && lane == 0;
    float* cbuf = reinterpret_cast<float*>(smem + L::kConstOffset);
    for (int c = t; c < 512; c += 256)
      cbuf[c] = c < 256 ? (args.bias ? args.bias[n0 + c] : 0.0f) : (args.ls1 ? args.ls1[n0 + c - 256] : 1.0f);
    named_bar_sync(1, 256);
    bool ok = mbar_wait(tfull_bar, 0, abort_flag, err, kDevTimeoutConsumer) && !*abort_flag;
    ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective
    for (int pass = 0; pass < 2; ++pass) {
      const int mp = m0 + pass * kBM;
      if (pass == 1) {
        // Pass 0's stores have read this half's staging tiles.
        if (store_thread) bulk_wait_all_read();
        named_bar_sync(2 + half, 128);
      }
      if (ok) {
        tc_fence_after();
#pragma unroll 1
        for (int j = 0; j < 4; ++j) {
          const int chunk = half * 4 + j;  // 32 columns
          float x[32];
          tmem_ld32(tmem + pass * 256 + chunk * 32 + (static_cast<uint32_t>(quad * 32) << 16), x);
          const float* bias = cbuf + chunk * 32;
          const float* scale = cbuf + 256 + chunk * 32;
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] = (x[i] + bias[i]) * scale[i];
          const uint32_t tile = base_u32 + chunk * kOutTileBytes;
#pragma unroll
          for (int c = 0; c < 8; ++c)
            st_shared_v4(tile + sw128_offset(row, c),
                         make_uint4(__float_as_uint(x[4 * c]), __float_as_uint(x[4 * c + 1]),
                                    __float_as_uint(x[4 * c + 2]), __float_as_uint(x[4 * c + 3])));
        }
      }
      fence_proxy_async_smem();  // the staged tiles are read by the TMA stores
      named_bar_sync(2 + half, 128);
      if (ok && mp < M && store_thread) {
        for (int j = 0; j < 4; ++j) {
          const int chunk = half * 4 + j;
          if (reduce)
            tma_reduce_add_2d(&map_out, base_u32 + chunk * kOutTileBytes, n0 + chunk * 32, mp);
          else
            tma_store_2d(&map_out, base_u32 + chunk * kOutTileBytes, n0 + chunk * 32, mp);
        }
        bulk_commit_group();
      }
    }
    if (store_thread) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (*abort_flag)
      for (int kb = *consumed; kb < *issued; ++kb) drain_wait(full_bar(kb % L::kStages), (kb / L::kStages) & 1);
    if (*mma_started) drain_wait(tfull_bar, 0);
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// 256 x 256 tiles in one wave when the call has between two thirds of and as many
// tiles as SMs (measured on B200: 123 tiles of the DA3 window 24.6 vs 26.7 us, fc2
// 51.7 vs 61.3 us; 63 tiles 22.7 vs 20.4 us, slower than the persistent kernel), N is a
// multiple of 256 and the residual, if any, is the output itself; otherwise the
// caller takes the persistent kernel.
cudaError_t launch_wide_proj(const __nv_bfloat16* a, const __nv_bfloat16* w_t, int M, int N, int K,
                             const ProjEpilogueArgs& args, int* err, cudaStream_t st, bool* used) {
  *used = false;
  if (N % 256 != 0 || K % kBK != 0 || K <= 0 || (args.residual && args.residual != args.out)) return cudaSuccess;
  const int n_tiles_n = N / 256;
  const int64_t tiles = static_cast<int64_t>((M + 2 * kBM - 1) / (2 * kBM)) * n_tiles_n;
  const int sms = device_sms();
  if (tiles > sms || 3 * tiles < 2 * sms) return cudaSuccess;
  CUtensorMap map_a, map_b, map_out;
  if (!encode_tma_2d_bf16(&map_a, a, K, M, kBK, 2 * kBM) || !encode_tma_2d_bf16(&map_b, w_t, K, N, kBK, 256) ||
      !encode_tma_2d_f32(&map_out, args.out, N, M, 32, kBM))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(gemm_bf16_wide_proj, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       WideSmem::kLaunchBytes);
  if (e != cudaSuccess) return e;
  gemm_bf16_wide_proj<<<static_cast<int>(tiles), kGemmThreads, WideSmem::kLaunchBytes, st>>>(
      map_a, map_b, map_out, args, M, K, n_tiles_n, args.residual ? 1 : 0, err);
  *used = true;
  return cudaGetLastError();
}

bool gemm_per_tile() {
  static const bool per_tile = std::getenv("VA_GEMM_PER_TILE") != nullptr;
  return per_tile;
}

// One place picks the kernel form for every GEMM of the path.
template <int BN, int STAGES_TILE, int MT, int STAGES_PERSIST, int CP, class Epi>
cudaError_t run_gemm(const __nv_bfloat16* a, const __nv_bfloat16* b, int M, int N, int K, const Epi& epi,
                     int* err, cudaStream_t st) {
  if (gemm_per_tile()) return launch_gemm<BN, STAGES_TILE>(a, b, M, N, K, epi, err, st);
  if constexpr (MT == 2) {
    // 256-row tiles only when they still fill every SM; a short call (one chunk of
    // the host pipeline, one rank's slice) keeps twice as many 128-row tiles.
    if (static_cast<int64_t>((M + 2 * kBM - 1) / (2 * kBM)) * (N / BN) < device_sms())
      return launch_gemm_persistent<BN, 1, 4, 1>(a, b, M, N, K, epi, err, st);
  }
  return launch_gemm_persistent<BN, MT, STAGES_PERSIST, CP>(a, b, M, N, K, epi, err, st);
}

}  // namespace

cudaError_t launch_qkv_gemm(const __nv_bfloat16* x, const __nv_bfloat16* w_qkv_t, int rows,
                            int embed, const QkvEpilogueArgs& epi, int* err, cudaStream_t st) {
  if (embed % 256 != 0 || epi.embed != embed || epi.rows != rows) return cudaErrorInvalidValue;
  QkvEpilogue e{};
  e.a = epi;
  if (!encode_tma_2d_bf16(&e.map_out[0], epi.q_out, embed, rows, 64, kBM) ||
      !encode_tma_2d_bf16(&e.map_out[1], epi.k_out, embed, rows, 64, kBM) ||
      !encode_tma_2d_bf16(&e.map_out[2], epi.v_out, embed, rows, 64, kBM))
    return cudaErrorInvalidValue;
  return run_gemm<256, 2, 1, 3, 1>(x, w_qkv_t, rows, 3 * embed, embed, e, err, st);
}

cudaError_t launch_fc1_gemm(const __nv_bfloat16* a, const __nv_bfloat16* w_t, int m, int n, int k,
                            const Fc1EpilogueArgs& epi, int* err, cudaStream_t st) {
  if (n % 256 != 0 || epi.rows != m || epi.hidden != n || !epi.bias) return cudaErrorInvalidValue;
  Fc1Epilogue e{};
  e.a = epi;
  if (!encode_tma_2d_bf16(&e.map_out, epi.out, n, m, 64, kBM)) return cudaErrorInvalidValue;
  return run_gemm<256, 2, 1, 3, 1>(a, w_t, m, n, k, e, err, st);
}

cudaError_t launch_proj_gemm(const __nv_bfloat16* a, const __nv_bfloat16* w_t, int m, int n, int k,
                             const ProjEpilogueArgs& epi, int* err, cudaStream_t st) {
  if (n % 128 != 0 || epi.embed != n || epi.rows != m) return cudaErrorInvalidValue;
  ProjEpilogue e{};
  e.a = epi;
  if (!encode_tma_2d_f32(&e.map_out, epi.out, n, m, 32, kBM)) return cudaErrorInvalidValue;
  if (!gemm_per_tile()) {
    bool used = false;
    const cudaError_t w = launch_wide_proj(a, w_t, m, n, k, epi, err, st, &used);
    if (w != cudaSuccess || used) return w;
  }
  if (epi.residual && !gemm_per_tile()) {
    if (!encode_tma_2d_f32(&e.map_res, epi.residual, n, m, 32, kBM)) return cudaErrorInvalidValue;
    e.res_staged = 1;
  }
  return run_gemm<128, 3, 2, 4, 2>(a, w_t, m, n, k, e, err, st);
}

cudaError_t launch_patch_gemm(const __nv_bfloat16* a, const __nv_bfloat16* w_t, int k,
                              const PatchEpilogueArgs& epi, int* err, cudaStream_t st) {
  if (epi.rows <= 0 || epi.n_patches <= 0 || epi.embed % 128 != 0 || k % kBK != 0 || !epi.bias ||
      !epi.pos || !epi.out || epi.n_tok != epi.n_special + epi.n_patches || epi.rows % epi.n_patches)
    return cudaErrorInvalidValue;
  PatchEpilogue e{};
  e.a = epi;
  const int views = epi.rows / epi.n_patches;
  if (!encode_tma_3d_f32_strided(&e.map_out, epi.out + static_cast<size_t>(epi.n_special) * epi.embed,
                                 epi.embed, epi.n_patches, views, static_cast<uint64_t>(epi.embed) * 4,
                                 static_cast<uint64_t>(epi.n_tok) * epi.embed * 4, 32, kBM, 1))
    return cudaErrorInvalidValue;
  // K = 640: a short main loop per tile, so the epilogue (position reads, row stores)
  // bounds it; one column pass keeps the epilogue to two passes per tile.
  return run_gemm<128, 3, 2, 3, 1>(a, w_t, epi.rows, epi.embed, k, e, err, st);
}

}  // namespace va
