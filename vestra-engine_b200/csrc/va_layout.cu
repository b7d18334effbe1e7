// Bandwidth-bound layout kernels of the attention path, plus TMA map encoding.
//
//   ln_cast      LN1 (vit_block.rs:696-714, optional) fused with the F32 -> bf16 cast
//                of the token rows that feed the QKV UMMA.  One warp per token row,
//                float4 loads, warp-shuffle mean/variance, 8-byte bf16 stores.
//   prep_heads   Op::Attention operand preparation (cpu_backend.rs:251-296): per
//                (head, token) LayerNorm over head_dim at qk_norm_eps, then 2D RoPE,
//                then bf16 token-major; one warp per row, two channels per lane.
//   camera_inject  camera-token slots before block alt_start (backbone.rs:746-768).
//   permute_views  view-order permutation (engine.rs:198-205 restore, backbone.rs:218-224).
//   patchify / pos_interp / token_specials  the token input side (patch_embed.rs:53-133,
//                pos_embed.rs:122-172, :254-300): NCHW images to bf16 patch rows for
//                the projection GEMM, the bicubic position table, the CLS and
//                register rows.
#include <cudaTypedefs.h>

#include <mutex>

#include "va_internal.h"
#include "va_ptx.cuh"

namespace va {

// ---------------------------------------------------------------------------
// TMA tensor maps
// ---------------------------------------------------------------------------
namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool get_encode() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode != nullptr;
}
}  // namespace

namespace {
PFN_cuStreamWriteValue32_v11070 g_write32 = nullptr;
std::once_flag g_write32_once;
PFN_cuStreamWriteValue64_v11070 g_write64 = nullptr;
std::once_flag g_write64_once;
}  // namespace

bool stream_write_u32(cudaStream_t st, int* addr, uint32_t value) {
  std::call_once(g_write32_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuStreamWriteValue32", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_write32 = reinterpret_cast<PFN_cuStreamWriteValue32_v11070>(fn);
  });
  if (!g_write32 || !addr) return false;
  // Default flags: the write is preceded by a memory fence over the stream's earlier work.
  return g_write32(reinterpret_cast<CUstream>(st), reinterpret_cast<CUdeviceptr>(addr), value,
                   CU_STREAM_WRITE_VALUE_DEFAULT) == CUDA_SUCCESS;
}

bool stream_write_u64(cudaStream_t st, unsigned long long* addr, unsigned long long value) {
  std::call_once(g_write64_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuStreamWriteValue64", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_write64 = reinterpret_cast<PFN_cuStreamWriteValue64_v11070>(fn);
  });
  if (!g_write64 || !addr) return false;
  // Default flags: the write is preceded by a memory fence over the stream's earlier work.
  return g_write64(reinterpret_cast<CUstream>(st), reinterpret_cast<CUdeviceptr>(addr), value,
                   CU_STREAM_WRITE_VALUE_DEFAULT) == CUDA_SUCCESS;
}

bool encode_tma_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                        uint32_t box_inner, uint32_t box_outer) {
  if (!get_encode() || base == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (inner * 2) % 16 != 0) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * 2};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_tma_2d_f32(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                       uint32_t box_inner, uint32_t box_outer) {
  if (!get_encode() || base == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (inner * 4) % 16 != 0) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * 4};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_tma_3d_f32_strided(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1,
                               uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                               uint32_t b0, uint32_t b1, uint32_t b2) {
  if (!get_encode() || base == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (d0 * 4) % 16 != 0 || stride1_bytes % 16 ||
      stride2_bytes % 16)
    return false;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  const cuuint32_t box[3] = {b0, b1, b2};
  const cuuint32_t estr[3] = {1, 1, 1};
  return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_tma_3d_bf16(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                        uint32_t b0, uint32_t b1, uint32_t b2) {
  if (!get_encode() || base == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (d0 * 2) % 16 != 0) return false;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {d0 * 2, d0 * d1 * 2};
  const cuuint32_t box[3] = {b0, b1, b2};
  const cuuint32_t estr[3] = {1, 1, 1};
  return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ---------------------------------------------------------------------------
// LN1 + cast
// ---------------------------------------------------------------------------
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// E % 128 == 0; each lane owns E/128 float4 groups of the row.
template <int kGroups>
__global__ void __launch_bounds__(256) ln_cast_kernel(const float* __restrict__ x,
                                                      const float* __restrict__ g,
                                                      const float* __restrict__ b, float eps,
                                                      int rows, int embed,
                                                      __nv_bfloat16* __restrict__ y) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * embed);
  float4 v[kGroups];
#pragma unroll
  for (int i = 0; i < kGroups; ++i) v[i] = __ldg(xr + i * 32 + lane);
  if (g != nullptr) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kGroups; ++i) s += v[i].x + v[i].y + v[i].z + v[i].w;
    const float mean = warp_sum(s) / embed;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < kGroups; ++i) {
      const float a = v[i].x - mean, bb = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
      q += a * a + bb * bb + c * c + d * d;
    }
    const float inv = 1.0f / sqrtf(warp_sum(q) / embed + eps);
    const float4* g4 = reinterpret_cast<const float4*>(g);
    const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
    for (int i = 0; i < kGroups; ++i) {
      const float4 gg = __ldg(g4 + i * 32 + lane), bb = __ldg(b4 + i * 32 + lane);
      v[i].x = (v[i].x - mean) * inv * gg.x + bb.x;
      v[i].y = (v[i].y - mean) * inv * gg.y + bb.y;
      v[i].z = (v[i].z - mean) * inv * gg.z + bb.z;
      v[i].w = (v[i].w - mean) * inv * gg.w + bb.w;
    }
  }
  uint2* yr = reinterpret_cast<uint2*>(y + static_cast<size_t>(row) * embed);
#pragma unroll
  for (int i = 0; i < kGroups; ++i)
    yr[i * 32 + lane] = make_uint2(pack_bf16x2(v[i].x, v[i].y), pack_bf16x2(v[i].z, v[i].w));
}

// One warp per (head, token) row of 64 channels; lane owns channels 2*lane, 2*lane+1.
__global__ void __launch_bounds__(256) prep_heads_kernel(
    const float* __restrict__ x, int rows_total, const float* __restrict__ g,
    const float* __restrict__ b, float eps, const int2* __restrict__ pos, int n,
    const float2* __restrict__ cs, int pairing, __nv_bfloat16* __restrict__ y, bool out_f16) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows_total) return;
  const float2 v = __ldg(reinterpret_cast<const float2*>(x + static_cast<size_t>(row) * 64) + lane);
  float a0 = v.x, a1 = v.y;
  if (g != nullptr) {
    const float mean = warp_sum(a0 + a1) * (1.0f / 64.0f);
    const float d0 = a0 - mean, d1 = a1 - mean;
    const float inv = 1.0f / sqrtf(warp_sum(d0 * d0 + d1 * d1) * (1.0f / 64.0f) + eps);
    a0 = d0 * inv * __ldg(g + 2 * lane) + __ldg(b + 2 * lane);
    a1 = d1 * inv * __ldg(g + 2 * lane + 1) + __ldg(b + 2 * lane + 1);
  }
  if (pos != nullptr) {
    const int t = row % n;
    const int2 p = pos[t];
    // channel c = 2*lane + e lives in half c/32 (0 = y, 1 = x), index c%32 in it.
    // Rotate-half partners (i, i+16) are channel c^16 = component e of lane^8.
    const float sw0 = __shfl_xor_sync(0xffffffffu, a0, 8);
    const float sw1 = __shfl_xor_sync(0xffffffffu, a1, 8);
    float out[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int c = 2 * lane + e;
      const int half = c >> 5;
      const int i = c & 31;
      const int pp = half == 0 ? p.x : p.y;
      const float me = e == 0 ? a0 : a1;
      float partner, sgn;
      int f;
      if (pairing == 0) {
        partner = e == 0 ? sw0 : sw1;
        f = i & 15;
        sgn = (i < 16) ? -1.f : 1.f;
      } else {
        // pairs (2k, 2k+1): the partner is the other channel of this lane
        partner = e == 0 ? a1 : a0;
        f = i >> 1;
        sgn = (e == 0) ? -1.f : 1.f;
      }
      const float2 cc = __ldg(cs + pp * 16 + f);
      out[e] = me * cc.x + sgn * partner * cc.y;
    }
    a0 = out[0];
    a1 = out[1];
  }
  // [H][n][64] -> token-major [n][H*64]
  const int heads = rows_total / n;
  const int h = row / n, t = row - h * n;
  reinterpret_cast<uint32_t*>(y + (static_cast<size_t>(t) * heads + h) * 64)[lane] =
      out_f16 ? f16x2_from_f32(a0, a1) : pack_bf16x2(a0, a1);
}

// first_is_reference: view 0 of this buffer is the window's view 0 (reference
// slot); a rank whose slice starts later gives every one of its views the source slot.
__global__ void camera_inject_kernel(float* tokens, const float* cam, int views,
                                     int tokens_per_view, int embed, int first_is_reference) {
  const int view = blockIdx.x;
  const float* src = cam + ((view > 0 || !first_is_reference) ? embed : 0);
  float* dst = tokens + static_cast<size_t>(view) * tokens_per_view * embed;
  for (int c = threadIdx.x; c < embed; c += blockDim.x) dst[c] = src[c];
}

__global__ void permute_views_kernel(const float4* src, float4* dst, const int* order,
                                     int64_t view_vec4) {
  const int view = blockIdx.y;
  const float4* s = src + static_cast<int64_t>(order[view]) * view_vec4;
  float4* d = dst + static_cast<int64_t>(view) * view_vec4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < view_vec4;
       i += (int64_t)gridDim.x * blockDim.x)
    d[i] = s[i];
}

// Patch rows for the projection GEMM (patch_embed.rs:53-133: a conv with
// kernel = stride = patch and no padding is one GEMM over these rows).  Thread =
// 8 consecutive features of one patch row (one 16-byte store).  kPatch > 0 fixes
// the patch size at compile time so the feature -> (c, ky, kx) split is
// multiply-shift arithmetic; kPatch = 0 reads it from `patch`.  32-bit indices
// (the launcher checks the range).
template <int kPatch>
__global__ void patchify_kernel(const float* __restrict__ img, int views, int height, int width,
                                int patch_rt, int kp_rt, __nv_bfloat16* __restrict__ rows) {
  const int patch = kPatch > 0 ? kPatch : patch_rt;
  const int kp = kPatch > 0 ? (3 * kPatch * kPatch + 63) / 64 * 64 : kp_rt;
  const int gw = width / patch, n_patches = (height / patch) * gw;
  const int vec_per_row = kp / 8;
  const int total = views * n_patches * vec_per_row;
  const int pp = patch * patch, features = 3 * pp;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int m = i / vec_per_row;
    const int k0 = (i - m * vec_per_row) * 8;
    uint4 u = make_uint4(0, 0, 0, 0);
    if (k0 < features) {
      const int view = m / n_patches, p = m - view * n_patches;
      const int py = p / gw, px = p - py * gw;
      const float* base = img + (static_cast<size_t>(view) * 3 * height + py * patch) * width + px * patch;
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int k = k0 + e;
        v[e] = 0.0f;
        if (k < features) {
          const int c = k / pp, rem = k - c * pp;
          const int ky = rem / patch, kx = rem - ky * patch;
          v[e] = __ldg(base + (static_cast<size_t>(c) * height + ky) * width + kx);
        }
      }
      u.x = pack_bf16x2(v[0], v[1]);
      u.y = pack_bf16x2(v[2], v[3]);
      u.z = pack_bf16x2(v[4], v[5]);
      u.w = pack_bf16x2(v[6], v[7]);
    }
    reinterpret_cast<uint4*>(rows)[i] = u;
  }
}

// Band form of the same, for the usual shapes: one CTA per (view, row of patches)
// reads the band's 3 x kPatch image rows once, coalesced, into shared memory, then
// writes the band's gw patch rows as 16-byte groups of 8 features (thread = one
// group of one patch, patches fastest: two-way bank conflicts at most).  The last
// `views` CTAs write each view's special rows instead (CLS + its position,
// registers), which saves a launch.
template <int kPatch>
__global__ void __launch_bounds__(256) patchify_band_kernel(
    const float* __restrict__ img, int views, int height, int width, int kp,
    __nv_bfloat16* __restrict__ rows, const float* __restrict__ cls, const float* __restrict__ pos,
    const float* __restrict__ regs, int n_register, int n_tok, int embed, float* __restrict__ tokens) {
  extern __shared__ float band[];  // [3 * kPatch][width]
  constexpr int kPP = kPatch * kPatch, kFeat = 3 * kPP;
  const int gh = height / kPatch, gw = width / kPatch;
  const int b = blockIdx.x;
  if (b >= views * gh) {
    const int view = b - views * gh;
    float* dst = tokens + static_cast<size_t>(view) * n_tok * embed;
    for (int i = threadIdx.x; i < (1 + n_register) * embed; i += blockDim.x) {
      const int row = i / embed, c = i - row * embed;
      dst[i] = row == 0 ? __fadd_rn(cls[c], pos[c]) : regs[static_cast<size_t>(row - 1) * embed + c];
    }
    return;
  }
  const int view = b / gh, py = b - view * gh;
  // The band's rows are contiguous per channel: channel c starts at image row
  // py*kPatch and spans kPatch*width floats.  Eight loads per thread are in flight
  // before their shared-memory stores.
  const int chan_f4 = kPatch * width / 4, total_f4 = 3 * chan_f4;
  constexpr int kUnroll = 8;
  for (int i0 = threadIdx.x; i0 < total_f4; i0 += blockDim.x * kUnroll) {
    float4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i < total_f4) {
        const int c = i / chan_f4, j = i - c * chan_f4;
        v[u] = __ldg(reinterpret_cast<const float4*>(
                         img + ((static_cast<size_t>(view) * 3 + c) * height + py * kPatch) * width) + j);
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i < total_f4) reinterpret_cast<float4*>(band)[i] = v[u];
    }
  }
  __syncthreads();
  const int groups = kp / 8;
  __nv_bfloat16* out = rows + static_cast<size_t>(b) * gw * kp;  // patch rows of this band
  for (int i = threadIdx.x; i < gw * groups; i += blockDim.x) {
    const int g = i / gw, px = i - g * gw;
    const int k0 = g * 8;
    uint4 u = make_uint4(0, 0, 0, 0);
    if (k0 < kFeat) {
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int k = k0 + e;
        v[e] = 0.0f;
        if (k < kFeat) {
          const int c = k / kPP, rem = k - c * kPP;
          const int ky = rem / kPatch, kx = rem - ky * kPatch;
          v[e] = band[(c * kPatch + ky) * width + px * kPatch + kx];
        }
      }
      u.x = pack_bf16x2(v[0], v[1]);
      u.y = pack_bf16x2(v[2], v[3]);
      u.z = pack_bf16x2(v[4], v[5]);
      u.w = pack_bf16x2(v[6], v[7]);
    }
    *reinterpret_cast<uint4*>(out + static_cast<size_t>(px) * kp + k0) = u;
  }
}

// Keys' cubic convolution kernel with a = -0.75 (pos_embed.rs:73-83), every
// operation rounded separately so the table is bit-identical to an F32 CPU
// evaluation in the same order.
__device__ __forceinline__ float cubic_a075(float x) {
  x = fabsf(x);
  if (x < 1.0f) return __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(__fmul_rn(1.25f, x), 2.25f), x), x), 1.0f);
  if (x < 2.0f)
    return __fmul_rn(__fsub_rn(__fmul_rn(__fadd_rn(__fmul_rn(__fsub_rn(x, 5.0f), x), 8.0f), x), 4.0f),
                     -0.75f);
  return 0.0f;
}

// interpolate_pos_embed (pos_embed.rs:122-172): thread = one channel of one row.
__global__ void pos_interp_kernel(const float* __restrict__ src, int grid, int embed, int gh, int gw,
                                  float offset, float* __restrict__ out) {
  const int64_t total = static_cast<int64_t>(1 + gh * gw) * embed;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i / embed), ch = static_cast<int>(i - static_cast<int64_t>(row) * embed);
    if (row == 0) {
      out[i] = src[ch];
      continue;
    }
    const int o = row - 1, oy = o / gw, ox = o - oy * gw;
    const float m = static_cast<float>(grid);
    const float sx = __fdiv_rn(__fadd_rn(static_cast<float>(gw), offset), m);
    const float sy = __fdiv_rn(__fadd_rn(static_cast<float>(gh), offset), m);
    const float iy = __fsub_rn(__fdiv_rn(__fadd_rn(static_cast<float>(oy), 0.5f), sy), 0.5f);
    const float ix = __fsub_rn(__fdiv_rn(__fadd_rn(static_cast<float>(ox), 0.5f), sx), 0.5f);
    const float y0f = floorf(iy), x0f = floorf(ix);
    const int y0 = static_cast<int>(y0f), x0 = static_cast<int>(x0f);
    const float fy = __fsub_rn(iy, y0f), fx = __fsub_rn(ix, x0f);
    float acc = 0.0f;
#pragma unroll
    for (int dy = -1; dy <= 2; ++dy) {
      const float wy = cubic_a075(__fsub_rn(fy, static_cast<float>(dy)));
      const int yy = min(max(y0 + dy, 0), grid - 1);
#pragma unroll
      for (int dx = -1; dx <= 2; ++dx) {
        const float wx = cubic_a075(__fsub_rn(fx, static_cast<float>(dx)));
        const int xx = min(max(x0 + dx, 0), grid - 1);
        const float s = __ldg(src + (static_cast<size_t>(1 + yy * grid + xx)) * embed + ch);
        acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(wy, wx), s));
      }
    }
    out[i] = acc;
  }
}

// Special rows of every view (pos_embed.rs:254-300): CLS + its position, then the
// register tokens unchanged.
__global__ void token_specials_kernel(const float* __restrict__ cls, const float* __restrict__ pos,
                                      const float* __restrict__ registers, int n_tok, int embed,
                                      float* __restrict__ out) {
  const int view = blockIdx.x, row = blockIdx.y;
  float* dst = out + (static_cast<size_t>(view) * n_tok + row) * embed;
  for (int c = threadIdx.x; c < embed; c += blockDim.x)
    dst[c] = row == 0 ? __fadd_rn(cls[c], pos[c]) : registers[static_cast<size_t>(row - 1) * embed + c];
}

}  // namespace

cudaError_t launch_patchify(const float* img, int views, int height, int width, int patch, int kp,
                            __nv_bfloat16* rows, cudaStream_t st) {
  if (!img || !rows || views <= 0 || patch <= 0 || height % patch || width % patch || height <= 0 ||
      width <= 0 || kp % 8 || kp < 3 * patch * patch)
    return cudaErrorInvalidValue;
  const int64_t total = static_cast<int64_t>(views) * (height / patch) * (width / patch) * (kp / 8);
  if (total >= (int64_t{1} << 31) || static_cast<int64_t>(views) * 3 * height * width >= (int64_t{1} << 40))
    return cudaErrorInvalidValue;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 16));
  if (patch == 14 && kp == 640)
    patchify_kernel<14><<<blocks, 256, 0, st>>>(img, views, height, width, patch, kp, rows);
  else
    patchify_kernel<0><<<blocks, 256, 0, st>>>(img, views, height, width, patch, kp, rows);
  return cudaGetLastError();
}

bool patchify_band_fits(int width, int patch, int kp) {
  return patch == 14 && kp == 640 && width % 4 == 0 &&
         static_cast<int64_t>(3) * patch * width * 4 <= kPatchBandMaxSmem;
}

cudaError_t launch_patchify_band(const float* img, int views, int height, int width, int patch, int kp,
                                 __nv_bfloat16* rows, const float* cls, const float* pos,
                                 const float* registers, int n_register, int n_tok, int embed,
                                 float* tokens, cudaStream_t st) {
  if (!img || !rows || !cls || !pos || !tokens || views <= 0 || height <= 0 || height % patch ||
      width % patch || !patchify_band_fits(width, patch, kp) || (reinterpret_cast<uintptr_t>(img) & 15) ||
      (n_register > 0 && !registers) ||
      n_tok != 1 + n_register + (height / patch) * (width / patch))
    return cudaErrorInvalidValue;
  const int smem = 3 * patch * width * 4;
  auto kern = patchify_band_kernel<14>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kern<<<views * (height / patch) + views, 256, smem, st>>>(img, views, height, width, kp, rows, cls, pos,
                                                            registers, n_register, n_tok, embed, tokens);
  return cudaGetLastError();
}

cudaError_t launch_pos_interp(const float* pos_embed, int grid, int embed, int gh, int gw,
                              float interp_offset, float* out, cudaStream_t st) {
  if (!pos_embed || !out || grid <= 0 || embed <= 0 || gh <= 0 || gw <= 0) return cudaErrorInvalidValue;
  const int64_t total = static_cast<int64_t>(1 + gh * gw) * embed;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 16));
  pos_interp_kernel<<<blocks, 256, 0, st>>>(pos_embed, grid, embed, gh, gw, interp_offset, out);
  return cudaGetLastError();
}

cudaError_t launch_token_specials(const float* cls, const float* pos, const float* registers,
                                  int n_register, int views, int n_tok, int embed, float* out,
                                  cudaStream_t st) {
  if (!cls || !pos || !out || views <= 0 || n_register < 0 || (n_register > 0 && !registers) ||
      n_tok <= n_register)
    return cudaErrorInvalidValue;
  token_specials_kernel<<<dim3(views, 1 + n_register), 256, 0, st>>>(cls, pos, registers, n_tok, embed, out);
  return cudaGetLastError();
}

cudaError_t launch_ln_cast(const float* x, const float* g, const float* b, float eps, int rows,
                           int embed, __nv_bfloat16* y, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const dim3 grid((rows + 7) / 8);
  switch (embed) {
    case 256: ln_cast_kernel<2><<<grid, 256, 0, st>>>(x, g, b, eps, rows, embed, y); break;
    case 512: ln_cast_kernel<4><<<grid, 256, 0, st>>>(x, g, b, eps, rows, embed, y); break;
    case 768: ln_cast_kernel<6><<<grid, 256, 0, st>>>(x, g, b, eps, rows, embed, y); break;
    case 1024: ln_cast_kernel<8><<<grid, 256, 0, st>>>(x, g, b, eps, rows, embed, y); break;
    case 1536: ln_cast_kernel<12><<<grid, 256, 0, st>>>(x, g, b, eps, rows, embed, y); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_prep_heads(const float* x, int heads, int n, const float* g, const float* b,
                              float eps, const int2* pos, const float2* rope_cs, int rope_pairing,
                              __nv_bfloat16* y, cudaStream_t st, bool out_f16) {
  const int total = heads * n;
  if (total <= 0) return cudaSuccess;
  prep_heads_kernel<<<(total + 7) / 8, 256, 0, st>>>(x, total, g, b, eps, pos, n, rope_cs,
                                                     rope_pairing, y, out_f16);
  return cudaGetLastError();
}

cudaError_t launch_camera_inject(float* tokens, const float* cam, int views, int tokens_per_view,
                                 int embed, cudaStream_t st, bool first_is_reference) {
  if (views <= 0) return cudaSuccess;
  camera_inject_kernel<<<views, 256, 0, st>>>(tokens, cam, views, tokens_per_view, embed,
                                              first_is_reference ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_permute_views(const float* src, float* dst, const int* order, int views,
                                 int64_t view_elems, cudaStream_t st) {
  if (views <= 0 || view_elems % 4 != 0) return cudaErrorInvalidValue;
  const int64_t v4 = view_elems / 4;
  dim3 grid(static_cast<unsigned>(std::min<int64_t>((v4 + 255) / 256, 1024)), views);
  permute_views_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const float4*>(src),
                                             reinterpret_cast<float4*>(dst), order, v4);
  return cudaGetLastError();
}

// Capture of one out layer (backbone.rs:1139-1179), one warp per patch row:
//   cat_token: feat[v][t] = [local_x row | LN_norm(x row)] (2E), cam[v] = [local_x row 0 | x row 0]
//   otherwise: feat[v][t] = LN_norm(x row) (E),              cam[v] = x row 0
// for the n - n_special patch rows t of every view v; LN with eps over E.
__global__ void capture_kernel(const float* __restrict__ x, const float* __restrict__ local_x,
                               const float* __restrict__ g, const float* __restrict__ b, float eps,
                               int views, int n, int n_special, int E, int cat, float* feat,
                               float* cam) {
  const int n_patch = n - n_special;
  const int64_t task = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int width = cat ? 2 * E : E;
  if (task < static_cast<int64_t>(views) * n_patch) {
    const int v = static_cast<int>(task / n_patch), t = static_cast<int>(task % n_patch);
    const float* xr = x + (static_cast<int64_t>(v) * n + n_special + t) * E;
    float* dst = feat + task * width;
    float s = 0.f;
    for (int c = lane; c < E; c += 32) s += xr[c];
    const float mean = warp_sum(s) / E;
    float q = 0.f;
    for (int c = lane; c < E; c += 32) {
      const float d = xr[c] - mean;
      q += d * d;
    }
    const float inv = 1.0f / sqrtf(warp_sum(q) / E + eps);
    float* nd = cat ? dst + E : dst;
    for (int c = lane; c < E; c += 32) nd[c] = (xr[c] - mean) * inv * g[c] + b[c];
    if (cat) {
      const float* lr = local_x + (static_cast<int64_t>(v) * n + n_special + t) * E;
      for (int c = lane; c < E; c += 32) dst[c] = lr[c];
    }
  } else if (task < static_cast<int64_t>(views) * n_patch + views) {
    const int v = static_cast<int>(task - static_cast<int64_t>(views) * n_patch);
    const float* xr = x + static_cast<int64_t>(v) * n * E;
    float* dst = cam + static_cast<int64_t>(v) * width;
    if (cat) {
      const float* lr = local_x + static_cast<int64_t>(v) * n * E;
      for (int c = lane; c < E; c += 32) dst[c] = lr[c];
      for (int c = lane; c < E; c += 32) dst[E + c] = xr[c];
    } else {
      for (int c = lane; c < E; c += 32) dst[c] = xr[c];
    }
  }
}

cudaError_t launch_capture(const float* x, const float* local_x, const float* g, const float* b,
                           float eps, int views, int n, int n_special, int E, int cat, float* feat,
                           float* cam, cudaStream_t st) {
  const int64_t tasks = static_cast<int64_t>(views) * (n - n_special) + views;
  const int per_block = 8;
  capture_kernel<<<static_cast<unsigned>((tasks + per_block - 1) / per_block), 32 * per_block, 0, st>>>(
      x, local_x, g, b, eps, views, n, n_special, E, cat, feat, cam);
  return cudaGetLastError();
}

// Failure-detection self-test: one thread waits on an mbarrier that nothing
// arrives on, through the same bounded wait the pipelined kernels use, so the
// wait gives up after limit_ns and writes kDevTimeoutConsumer into the device
// error word; the kernel then returns normally.
__global__ void bounded_wait_selftest_kernel(unsigned long long limit_ns, int* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait_for(b, 0, &abort_flag, err, kDevTimeoutConsumer, limit_ns);
  __syncthreads();
}

// Flags of the epilogue-store K'/V exchange, one warp: lane p publishes this rank's
// flag value to peer p (system-scope release, no wait).  The QKV kernel before it
// on the stream stored the rows; the fence and the release order those stores
// before the flag, and the peer's attention kernel reads the flag with acquire.
__global__ void peer_flags_kernel(PeerFlagArgs a) {
  const int p = threadIdx.x;
  if (p < a.npeer) {
    __threadfence_system();
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(a.peer_flag[p]), "l"(a.value) : "memory");
  }
}

cudaError_t launch_peer_flags(const PeerFlagArgs& a, cudaStream_t st) {
  if (a.npeer < 0 || a.npeer > kMaxPeers) return cudaErrorInvalidValue;
  if (a.npeer == 0) return cudaSuccess;
  peer_flags_kernel<<<1, 32, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_bounded_wait_selftest(unsigned long long limit_ns, int* err, cudaStream_t st) {
  bounded_wait_selftest_kernel<<<1, 32, 0, st>>>(limit_ns, err);
  return cudaGetLastError();
}

}  // namespace va
