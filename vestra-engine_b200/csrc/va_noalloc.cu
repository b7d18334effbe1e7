// Op::Attention for callers that must not allocate device memory.
//
// Some callers of this library cannot call cudaMalloc: a serving process that
// reserves all device memory for its own pool up front, or an engine whose
// block loop must never hit an allocation failure (or the device-wide
// synchronisation a cudaMalloc/cudaFree can cause) halfway through a model.
// va_op_attention_noalloc gives them the Op::Attention computation with no
// allocation at all: the bf16 operand scratch lives in a fixed-size array in
// the library's own device memory, which every GPU that loads the library keeps
// until the process exits.  The caller passes inputs and outputs as usual.
//
// Limits and behaviour:
//   * heads * n * 64 <= kNoAllocMaxElems (2,097,152) per operand, i.e. 12 MiB of
//     scratch for Q, K and V together; larger requests return VA_ERR_CAPACITY.
//   * The first call on a device looks up the scratch's device address
//     (cudaGetSymbolAddress) with that device current; make that first call
//     before any stream capture.
//   * Every call shares the one scratch array, and it keeps the previous call's
//     contents: calls that overlap on the GPU (other streams, other host
//     threads) race and must be serialised by the caller.  Rows past n are
//     never read (the TMA boxes are bounded by n), and the device error word is
//     cleared at the start of every call.
//   * The call is synchronous: it waits for its stream and returns
//     VA_ERR_DEVICE if a kernel gave up on a bounded wait.
//   * RoPE positions are rounded half away from zero (f32::round, as the
//     reference's cpu_backend.rs:291-292 and the context entry points) and must lie
//     in [0, 65535] like theirs; a position outside that range makes the call
//     return VA_ERR_INVALID (checked on the device, so nothing is copied to the host).
#include <cmath>
#include <mutex>

#include "../../include/vestra_attn.h"
#include "va_internal.h"
#include "va_ptx.cuh"

namespace {

constexpr size_t kNoAllocMaxElems = size_t(1) << 21;  // per operand (bf16 elements)
constexpr int kBadPosition = va::kDevBadShape;        // error word: a position out of range

// freq^(-2i/32), i < 16, computed on the host in double.
struct InvFreq {
  double v[16];
};
constexpr int kMaxDevices = 64;

static __device__ __align__(256) __nv_bfloat16 g_noalloc_scratch[3 * kNoAllocMaxElems];
static __device__ __align__(256) int g_noalloc_err;

// Device addresses of the two symbols, looked up once per device.
struct DeviceSymbols {
  bool ready = false;
  __nv_bfloat16* scratch = nullptr;
  int* err = nullptr;
};
std::mutex g_mu;
DeviceSymbols g_symbols[kMaxDevices];

int device_symbols(DeviceSymbols* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return VA_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceSymbols& s = g_symbols[dev];
  if (!s.ready) {
    // The current device is `dev`: the addresses below belong to it.
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return VA_ERR_CUDA;
    s.scratch = static_cast<__nv_bfloat16*>(p);
    p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_err) != cudaSuccess || p == nullptr) return VA_ERR_CUDA;
    s.err = static_cast<int*>(p);
    s.ready = true;
  }
  *out = s;
  return VA_OK;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// [H][n][64] F32 -> optional per-row LayerNorm -> optional 2D RoPE -> token-major
// bf16 [n][H*64].  Positions come from a device F32 [n][2] table (rounded half away
// from zero, as in cpu_backend.rs:291-292) and the rotation angles
// pos * freq^(-2i/32) are formed here in double, like the context's host table, so
// the call needs no host-built table.  A position outside [0, 65535] sets *err.
__global__ void __launch_bounds__(256) noalloc_prep_kernel(
    const float* __restrict__ x, int rows_total, int n, const float* __restrict__ g,
    const float* __restrict__ b, float eps, const float* __restrict__ pos_yx, InvFreq inv_freq,
    int pairing, __nv_bfloat16* __restrict__ y, int* err) {
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
  const int heads = rows_total / n;
  const int h = row / n, t = row - h * n;
  if (pos_yx != nullptr) {
    const float py = roundf(__ldg(pos_yx + 2 * t)), px = roundf(__ldg(pos_yx + 2 * t + 1));
    if (!(py >= 0.f && py <= 65535.f && px >= 0.f && px <= 65535.f)) {  // NaN fails too
      if (lane == 0) atomicCAS(err, 0, kBadPosition);
      return;
    }
    const float sw0 = __shfl_xor_sync(0xffffffffu, a0, 8);  // rotate-half partner, channel c^16
    const float sw1 = __shfl_xor_sync(0xffffffffu, a1, 8);
    float out[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int c = 2 * lane + e;
      const int i = c & 31;
      const float p = (c >> 5) == 0 ? py : px;
      const float me = e == 0 ? a0 : a1;
      float partner, sgn;
      int f;
      if (pairing == 0) {
        partner = e == 0 ? sw0 : sw1;
        f = i & 15;
        sgn = (i < 16) ? -1.f : 1.f;
      } else {
        partner = e == 0 ? a1 : a0;
        f = i >> 1;
        sgn = (e == 0) ? -1.f : 1.f;
      }
      double s, co;
      sincos(static_cast<double>(p) * inv_freq.v[f], &s, &co);
      out[e] = me * static_cast<float>(co) + sgn * partner * static_cast<float>(s);
    }
    a0 = out[0];
    a1 = out[1];
  }
  reinterpret_cast<uint32_t*>(y + (static_cast<size_t>(t) * heads + h) * 64)[lane] =
      va::pack_bf16x2(a0, a1);
}

}  // namespace

extern "C" int va_op_attention_noalloc(const float* q, const float* k, const float* v, int heads,
                                       int64_t n, int head_dim, const float* qn_g,
                                       const float* qn_b, const float* kn_g, const float* kn_b,
                                       float qk_norm_eps, const float* pos_yx_dev, float freq,
                                       int rope_pairing, float* out, void* stream) {
  if (!q || !k || !v || !out || head_dim != 64 || heads <= 0 || n <= 0) return VA_ERR_INVALID;
  if ((qn_g == nullptr) != (qn_b == nullptr) || (kn_g == nullptr) != (kn_b == nullptr))
    return VA_ERR_INVALID;
  if (rope_pairing != 0 && rope_pairing != 1) return VA_ERR_INVALID;
  if (pos_yx_dev && !(freq > 0.0f)) return VA_ERR_INVALID;
  if (static_cast<size_t>(heads) * static_cast<size_t>(n) * 64 > kNoAllocMaxElems)
    return VA_ERR_CAPACITY;
  DeviceSymbols sym;
  int rc = device_symbols(&sym);
  if (rc != VA_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int rows = heads * static_cast<int>(n);
  __nv_bfloat16* qs = sym.scratch;
  __nv_bfloat16* ks = sym.scratch + kNoAllocMaxElems;
  __nv_bfloat16* vs = sym.scratch + 2 * kNoAllocMaxElems;
  if (cudaMemsetAsync(sym.err, 0, sizeof(int), st) != cudaSuccess) return VA_ERR_CUDA;
  InvFreq inv{};
  for (int i = 0; i < 16; ++i) inv.v[i] = std::pow(static_cast<double>(freq), -2.0 * i / 32.0);
  const dim3 grid((rows + 7) / 8);
  noalloc_prep_kernel<<<grid, 256, 0, st>>>(q, rows, static_cast<int>(n), qn_g, qn_b, qk_norm_eps,
                                            pos_yx_dev, inv, rope_pairing, qs, sym.err);
  noalloc_prep_kernel<<<grid, 256, 0, st>>>(k, rows, static_cast<int>(n), kn_g, kn_b, qk_norm_eps,
                                            pos_yx_dev, inv, rope_pairing, ks, sym.err);
  noalloc_prep_kernel<<<grid, 256, 0, st>>>(v, rows, static_cast<int>(n), nullptr, nullptr, 0.f,
                                            nullptr, inv, 0, vs, sym.err);
  if (cudaGetLastError() != cudaSuccess) return VA_ERR_CUDA;
  va::FlashArgs fa{};
  fa.q_count = static_cast<int>(n);
  fa.q_offset = 0;
  fa.kv_rows = static_cast<int>(n);
  fa.seg_len = 0;
  fa.heads = heads;
  fa.scale_log2 = static_cast<float>(1.0 / 8.0 * 1.4426950408889634);
  fa.out_mode = 1;
  fa.o_hnd = out;
  fa.embed = heads * 64;
  if (va::launch_flash(qs, ks, vs, fa, sym.err, st) != cudaSuccess) return VA_ERR_CUDA;
  int h_err = 0;
  if (cudaMemcpyAsync(&h_err, sym.err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return VA_ERR_CUDA;
  return h_err == 0 ? VA_OK : h_err == kBadPosition ? VA_ERR_INVALID : VA_ERR_DEVICE;
}
