// K2: fused flash attention for head_dim 64 on sm_100a (tcgen05 + TMEM + TMA).
//
// Semantics: per head and per independent segment of seg_len tokens,
//   O = softmax(Q K^T / sqrt(64)) V   (non-causal, FP32 online softmax),
// which is vestra_kernels::attention at vit_block.rs:951-953 over the flattened
// view-major sequence (global blocks: one segment of S*n tokens) or over each
// view (local blocks batched: S segments of n tokens, block-diagonal).
// Q and K arrive already QK-normalised and rotated (K1 epilogue, or the
// Op::Attention prep kernel).  All operands are bf16 token-major [rows][E]; the
// TMA box of head h is the 64-column slab [64h, 64h+64) (128 B per row), so a
// rank's queries can run against a key window gathered from other ranks.
//
// CTA = one (segment, head, pair of 128-query tiles).  10 warps:
//   warp 0      TMA producer: Q0/Q1 once, then K_j/V_j into a STAGES-deep ring
//   warp 1      TMEM owner + single-thread UMMA issuer
//   warps 2..5  softmax warpgroup for query tile 0 (thread = query row)
//   warps 6..9  softmax warpgroup for query tile 1
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,320) O1 [320,384).
// P_t (bf16x2-packed probabilities) overwrites the first 64 columns of S_t and
// feeds the PV UMMA straight from TMEM (A operand in TMEM), so P never touches
// shared memory.  The two query tiles ping-pong: while one warpgroup runs the
// softmax of KV tile j, the tensor core runs the other tile's PV(j) and QK(j+1).
//
// Per KV tile j and query tile t the issue order is PV_t(j-1) then QK_t(j); the
// commit that signals S_t(j) therefore also covers PV_t(j-1), so when a softmax
// warpgroup sees S_t(j) ready, O_t holds every earlier contribution and the
// columns of P_t(j-1) may be overwritten.  O_t is rescaled in TMEM by its own
// warpgroup when the running row max grows.
#include <math.h>

#include "va_internal.h"
#include "va_ptx.cuh"

namespace va {

namespace {

constexpr int kTileQ = 128;
constexpr int kTileK = 128;
constexpr int kHeadDim = 64;
constexpr int kStages = 3;
constexpr int kFlashThreads = 320;
constexpr uint32_t kTileBytes = kTileQ * kHeadDim * 2;  // 16 KB, one bf16 [128][64] tile
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColO0 = 256;

struct FlashSmem {
  static constexpr uint32_t kQ = 0;                              // Q0, Q1
  static constexpr uint32_t kK = 2 * kTileBytes;                 // K ring
  static constexpr uint32_t kV = kK + kStages * kTileBytes;      // V ring
  static constexpr uint32_t kBar = kV + kStages * kTileBytes;
  // barriers: q_full, kv_full[S], kv_empty[S], s_full[2], p_full[2], o_final[2]
  static constexpr uint32_t kNumBars = 1 + 2 * kStages + 6;
  static constexpr uint32_t kMisc = kBar + 8 * kNumBars;
  static constexpr uint32_t kBytes = kMisc + 64;
  static constexpr uint32_t kLaunchBytes = kBytes + 1024;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void drain(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) break;
  }
}

__global__ void __launch_bounds__(kFlashThreads, 1)
    flash_fwd_d64_kernel(const __grid_constant__ CUtensorMap map_q,
                         const __grid_constant__ CUtensorMap map_k,
                         const __grid_constant__ CUtensorMap map_v, FlashArgs fa, int* err) {
  using L = FlashSmem;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_u32);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int pair = blockIdx.x;
  const int head = blockIdx.y;
  const int seg = blockIdx.z;
  const bool global = fa.seg_len == 0;
  // Query rows of this CTA (in the local Q buffer) and the key range they see.
  const int q_seg0 = global ? 0 : seg * fa.seg_len;
  const int q_end = global ? fa.q_count : q_seg0 + fa.seg_len;
  const int q0 = q_seg0 + pair * 2 * kTileQ;
  const int k0 = global ? 0 : fa.q_offset + q_seg0;
  const int klen = global ? fa.kv_rows : fa.seg_len;
  const int nq = (q_end - q0) > kTileQ ? 2 : 1;  // query tiles with valid rows
  const int num_kv = (klen + kTileK - 1) / kTileK;
  const bool tail_mask = (num_kv * kTileK) != klen;
  const int col = head * kHeadDim;

  const uint32_t bar_q = base + L::kBar;
  auto bar_kv_full = [&](int s) { return base + L::kBar + 8u * (1 + s); };
  auto bar_kv_empty = [&](int s) { return base + L::kBar + 8u * (1 + kStages + s); };
  auto bar_s_full = [&](int t) { return base + L::kBar + 8u * (1 + 2 * kStages + t); };
  auto bar_p_full = [&](int t) { return base + L::kBar + 8u * (3 + 2 * kStages + t); };
  auto bar_o_final = [&](int t) { return base + L::kBar + 8u * (5 + 2 * kStages + t); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
  volatile int* kv_issued = reinterpret_cast<volatile int*>(smem + L::kMisc + 8);
  volatile int* kv_consumed = reinterpret_cast<volatile int*>(smem + L::kMisc + 12);
  volatile int* mma_done = reinterpret_cast<volatile int*>(smem + L::kMisc + 16);
  auto sQ = [&](int t) { return base + L::kQ + t * kTileBytes; };
  auto sK = [&](int s) { return base + L::kK + s * kTileBytes; };
  auto sV = [&](int s) { return base + L::kV + s * kTileBytes; };

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar_kv_full(s), 1);
      mbar_init(bar_kv_empty(s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar_s_full(t), 1);
      mbar_init(bar_p_full(t), 128);
      mbar_init(bar_o_final(t), 1);
    }
    *abort_flag = 0;
    *kv_issued = 0;
    *kv_consumed = 0;
    *mma_done = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_v);
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
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      // Every box starts inside the tensor; rows past its end are zero-filled.
      mbar_arrive_expect_tx(bar_q, nq * kTileBytes);
      tma_load_2d(sQ(0), &map_q, bar_q, col, q0);
      if (nq == 2) tma_load_2d(sQ(1), &map_q, bar_q, col, q0 + kTileQ);
      for (int j = 0; j < num_kv; ++j) {
        const int s = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        if (!mbar_wait(bar_kv_empty(s), ph ^ 1, abort_flag, err, kDevTimeoutProducer)) break;
        mbar_arrive_expect_tx(bar_kv_full(s), 2 * kTileBytes);
        tma_load_2d(sK(s), &map_k, bar_kv_full(s), col, k0 + j * kTileK);
        tma_load_2d(sV(s), &map_v, bar_kv_full(s), col, k0 + j * kTileK);
        *kv_issued = j + 1;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_bf16_f32(kTileQ, kTileK, false, false);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(kTileQ, kHeadDim, false, true);
      bool ok = mbar_wait(bar_q, 0, abort_flag, err, kDevTimeoutMma);
      auto issue_qk = [&](int t, int s) {
#pragma unroll
        for (int k = 0; k < kHeadDim / 16; ++k) {
          const uint64_t ad = sdesc_sw128(sQ(t) + k * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(sK(s) + k * 32, 16, 1024);
          umma_ss(tmem + kColS0 + t * 128, ad, bd, idesc_qk, k != 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int t, int s, bool acc) {
#pragma unroll
        for (int k = 0; k < kTileK / 16; ++k) {
          // B = V tile, MN-major: 16 keys per step = 16 rows of 128 B.
          const uint64_t bd = sdesc_sw128(sV(s) + k * 16 * 128, 8192, 1024);
          umma_ts(tmem + kColO0 + t * 64, tmem + kColS0 + t * 128 + k * 8, bd, idesc_pv,
                  (acc || k != 0) ? 1u : 0u);
        }
      };
      if (ok) ok = mbar_wait(bar_kv_full(0), 0, abort_flag, err, kDevTimeoutMma);
      if (ok) {
        *kv_consumed = 1;
        tc_fence_after();
        for (int t = 0; t < nq; ++t) {
          issue_qk(t, 0);
          tc_commit(bar_s_full(t));
        }
      }
      for (int j = 0; ok && j < num_kv; ++j) {
        const int s = j % kStages;
        for (int t = 0; t < nq && ok; ++t) {
          ok = mbar_wait(bar_p_full(t), j & 1, abort_flag, err, kDevTimeoutMma);
          if (!ok) break;
          tc_fence_after();
          issue_pv(t, s, j > 0);
          if (j + 1 < num_kv) {
            const int s1 = (j + 1) % kStages;
            if (t == 0) {
              ok = mbar_wait(bar_kv_full(s1), ((j + 1) / kStages) & 1, abort_flag, err,
                             kDevTimeoutMma);
              if (!ok) break;
              *kv_consumed = j + 2;
              tc_fence_after();
            }
            issue_qk(t, s1);
            tc_commit(bar_s_full(t));
          }
        }
        tc_commit(bar_kv_empty(s));
      }
      for (int t = 0; t < 2; ++t) tc_commit(bar_o_final(t));
      *mma_done = 1;
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int t = (warp - 2) >> 2;              // query tile of this warpgroup
    const int quad = warp & 3;                  // TMEM lane quadrant
    const int r = quad * 32 + lane;             // row inside the query tile
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + lane_off + kColS0 + t * 128;
    const uint32_t tO = tmem + lane_off + kColO0 + t * 64;
    const float sl2 = fa.scale_log2;
    if (t < nq) {
      float m = -INFINITY;  // running max, log2 domain (already multiplied by scale_log2)
      float l = 0.f;
      bool ok = true;
      for (int j = 0; j < num_kv; ++j) {
        ok = mbar_wait(bar_s_full(t), j & 1, abort_flag, err, kDevTimeoutConsumer);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        float s[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, s + c * 32);
        if (tail_mask && j == num_kv - 1) {
          const int valid = klen - j * kTileK;
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c >= valid) s[c] = -INFINITY;
        }
        float mx = s[0];
#pragma unroll
        for (int c = 1; c < 128; ++c) mx = fmaxf(mx, s[c]);
        const float m_new = fmaxf(m, mx * sl2);
        const float alpha = ex2(m - m_new);  // 0 on the first tile (m = -inf)
        const float neg = -m_new;
        float sum = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float p0 = ex2(fmaf(s[c * 32 + 2 * i], sl2, neg));
            const float p1 = ex2(fmaf(s[c * 32 + 2 * i + 1], sl2, neg));
            sum += p0 + p1;
            pk[i] = pack_bf16x2(p0, p1);
          }
          tmem_st16(tS + c * 16, pk);
        }
        if (j > 0 && __any_sync(0xffffffffu, alpha < 1.0f)) {
          float o[64];
          tmem_ld32(tO, o);
          tmem_ld32(tO + 32, o + 32);
          uint32_t u[16];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
#pragma unroll
            for (int i = 0; i < 16; ++i) u[i] = __float_as_uint(o[c * 16 + i] * alpha);
            tmem_st16(tO + c * 16, u);
          }
        }
        tmem_wait_st();
        l = l * alpha + sum;
        m = m_new;
        tc_fence_before();
        mbar_arrive(bar_p_full(t));
      }
      bool fin = ok && mbar_wait(bar_o_final(t), 0, abort_flag, err, kDevTimeoutConsumer);
      fin = __all_sync(0xffffffffu, fin);
      if (fin) {
        tc_fence_after();
        float o[64];
        tmem_ld32(tO, o);
        tmem_ld32(tO + 32, o + 32);
        const int token = q0 + t * kTileQ + r;  // row of the local Q / O buffers
        if (token < q_end) {
          const float inv = 1.0f / l;
          if (fa.out_mode == 0) {
#pragma unroll
            for (int i = 0; i < 64; ++i) o[i] *= inv;
            uint4* d = reinterpret_cast<uint4*>(fa.o_tok + static_cast<size_t>(token) * fa.embed +
                                                head * kHeadDim);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              uint4 w;
              w.x = pack_bf16x2(o[8 * c + 0], o[8 * c + 1]);
              w.y = pack_bf16x2(o[8 * c + 2], o[8 * c + 3]);
              w.z = pack_bf16x2(o[8 * c + 4], o[8 * c + 5]);
              w.w = pack_bf16x2(o[8 * c + 6], o[8 * c + 7]);
              d[c] = w;
            }
          } else {
            float4* d = reinterpret_cast<float4*>(
                fa.o_hnd + (static_cast<size_t>(head) * fa.q_count + token) * kHeadDim);
#pragma unroll
            for (int c = 0; c < 16; ++c)
              d[c] = make_float4(o[4 * c] * inv, o[4 * c + 1] * inv, o[4 * c + 2] * inv,
                                 o[4 * c + 3] * inv);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) {
    // Drain copies and UMMAs still in flight before TMEM is released.
    if (*kv_consumed == 0) drain(bar_q, 0);
    for (int j = *kv_consumed; j < *kv_issued; ++j) drain(bar_kv_full(j % kStages), (j / kStages) & 1);
    if (*mma_done) drain(bar_o_final(0), 0);
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

cudaError_t launch_flash(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v,
                         const FlashArgs& fa, int* err, cudaStream_t st) {
  // Every TMA box must start inside its tensor: q rows [0, q_count), key rows
  // [q_offset + segment start, +seg_len) or [0, kv_rows).
  if (fa.q_count <= 0 || fa.kv_rows <= 0 || fa.heads <= 0 || fa.embed != fa.heads * kHeadDim ||
      fa.q_offset < 0 || fa.seg_len < 0)
    return cudaErrorInvalidValue;
  int segs = 1;
  if (fa.seg_len > 0) {
    if (fa.q_count % fa.seg_len != 0 || fa.q_offset % fa.seg_len != 0 ||
        static_cast<int64_t>(fa.q_offset) + fa.q_count > fa.kv_rows)
      return cudaErrorInvalidValue;
    segs = fa.q_count / fa.seg_len;
  }
  CUtensorMap mq, mk, mv;
  if (!encode_tma_2d_bf16(&mq, q, fa.embed, fa.q_count, kHeadDim, kTileQ) ||
      !encode_tma_2d_bf16(&mk, k, fa.embed, fa.kv_rows, kHeadDim, kTileK) ||
      !encode_tma_2d_bf16(&mv, v, fa.embed, fa.kv_rows, kHeadDim, kTileK))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(flash_fwd_d64_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       FlashSmem::kLaunchBytes);
  if (e != cudaSuccess) return e;
  const int span = fa.seg_len > 0 ? fa.seg_len : fa.q_count;
  dim3 grid((span + 2 * kTileQ - 1) / (2 * kTileQ), fa.heads, segs);
  flash_fwd_d64_kernel<<<grid, kFlashThreads, FlashSmem::kLaunchBytes, st>>>(mq, mk, mv, fa, err);
  return cudaGetLastError();
}

}  // namespace va
