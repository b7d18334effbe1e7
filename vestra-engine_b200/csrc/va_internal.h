// Internal launcher interface between the C-ABI layer (va_api.cu) and the
// kernels (va_gemm.cu, va_flash.cu, va_layout.cu).  Plain pointers and sizes;
// no torch types anywhere in the library.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

struct va_gguf;

namespace va {

// ---- QKV projection (K1): X[rows,E] bf16 x Wqkv^T -> Q,K,V token-major bf16 ----
constexpr int kMaxRanks = 8;
constexpr int kMaxPeers = kMaxRanks - 1;

struct QkvEpilogueArgs {
  const float* bias;                  // [3E]
  const float* q_g; const float* q_b;  // [64] QK-norm (nullptr: no QK-norm)
  const float* k_g; const float* k_b;
  float qk_eps;
  const int2* pos;                     // [rows] (y, x) integer positions (nullptr: no RoPE)
  const float2* rope_cs;               // [16][rope_npos] (cos, sin) of pos * base^(-2i/32), i-major
  int rope_npos;
  int rope_pairing;                    // 0 rotate-half, 1 interleaved
  __nv_bfloat16* q_out;                // [rows][E], head h at columns [64h, 64h+64)
  __nv_bfloat16* k_out;                // [rows][E] (may be a rank's slice of a gathered buffer)
  __nv_bfloat16* v_out;               // bf16, or f16 bits when v_f16
  int rows;
  int embed;
  int v_f16;                           // store V as f16 (the PV UMMA then runs in f16)
  // Direct K'/V exchange: the same rows of K' and V are also stored into these
  // peer GPUs' window buffers (their slice of this rank, over NVLink).
  int npeer = 0;
  __nv_bfloat16* peer_k[kMaxPeers] = {};
  __nv_bfloat16* peer_v[kMaxPeers] = {};
};

// MLP fc1 epilogue: + bias, exact GELU, bf16 out [rows][hidden].
struct Fc1EpilogueArgs {
  const float* bias;     // [hidden]
  __nv_bfloat16* out;    // [rows][hidden]
  int rows;
  int hidden;
};
cudaError_t launch_fc1_gemm(const __nv_bfloat16* a, const __nv_bfloat16* w_t, int m, int n, int k,
                            const Fc1EpilogueArgs& epi, int* err, cudaStream_t st);

// Flag writes of the epilogue-store K'/V exchange: after the QKV kernel's peer
// stores, value is written (system-scope release) to each peer's flag, with no
// wait: the attention kernels wait on their own flags.
struct PeerFlagArgs {
  unsigned long long* peer_flag[kMaxPeers];  // this rank's flag in each peer's flag array
  int npeer;
  unsigned long long value;
};
cudaError_t launch_peer_flags(const PeerFlagArgs& a, cudaStream_t st);

// ---- output projection (K3): O[rows,E] bf16 x Wp^T + b (* ls1) (+ residual) -> F32 ----
struct ProjEpilogueArgs {
  const float* bias;      // [E]
  const float* ls1;       // [E] or nullptr
  const float* residual;  // [rows,E] F32 or nullptr (may alias out)
  float* out;             // [rows,E] F32
  int rows;
  int embed;
};

// Patch projection epilogue: GEMM row m = patch p of view s (m = s*n_patches + p),
// written to token row s*n_tok + n_special + p as conv + bias + pos[1 + p].
struct PatchEpilogueArgs {
  const float* bias;  // [E]
  const float* pos;   // [(1 + n_patches)][E]: row 0 = CLS position, row 1 + p = patch p
  float* out;         // [views][n_tok][E]
  int rows;           // views * n_patches
  int n_patches;
  int n_tok;          // n_special + n_patches
  int n_special;
  int embed;
};

// ---- fused flash attention (K2) ----
// Default softmax variant (poly + 8 * form): form 3 (four threads per row, 20
// warps), every exponential on MUFU.
constexpr int kDefaultPolyPer8 = 24;
// Default for launches with the fixed exponent offset: form 10 (key split between
// MUFU and FMA-pipe warps, quadratic exp2 on the FMA pipe), KA = 64 + 8 * 1 = 72
// keys of every 128 on MUFU (the fastest split measured at S=12).
constexpr int kDefaultKeySplit = 10 * 8 + 1;
// The same softmax with one query tile per CTA and two CTAs per SM (form 15, KA = 72):
// the default for local attention (few key tiles per CTA, so a CTA's fill and drain
// are a large share of its time and the other CTA on the SM covers them) and for
// global launches whose query pairs fill 1.5 to 2 waves (one rank's half window).
constexpr int kDefaultKeySplit1 = 15 * 8 + 1;
// Q is [q_count][E] token-major (this rank's queries, the first of which is row
// q_offset of the key window); K and V are [kv_rows][E] token-major.
// seg_len == 0: global attention, every query sees all kv_rows keys.
// seg_len  > 0: local attention over independent segments of seg_len tokens;
//               q_offset and q_count are then multiples of seg_len.
struct FlashArgs {
  int q_count;
  int q_offset;
  int kv_rows;
  int seg_len;
  int heads;
  float scale_log2;       // (1/sqrt(64)) * log2(e)
  int out_mode;           // 0: token-major bf16 [q_count][E]; 1: head-major F32 [H][q_count][64]
  __nv_bfloat16* o_tok;
  float* o_hnd;
  int embed;
  int v_f16;              // 1: V holds f16 and P is formed in f16; 0: V and P are bf16
  // bf16 path: variant = poly + 8 * form (see launch_flash); < 0: the library default
  // (with fixed_offset kDefaultKeySplit1 for local attention and global launches of
  // 1.5 to 2 waves of query pairs, else kDefaultKeySplit; without it kDefaultPolyPer8)
  int poly_per8 = -1;
  // 1: exponents relative to 0 instead of the running row max (w20 kernel, bf16 P;
  // other forms ignore it).  Only for inputs with |q.k| * scale * log2(e) <= 64.
  int fixed_offset = 0;
  // Split-key tail of global attention (four-threads-per-row kernel only).  With
  // U = heads x query-pairs units and `sms` multiprocessors, the last U mod sms
  // units (the partial last wave) are each run as `splits` CTAs over disjoint key
  // ranges; their unnormalised partial results meet in part_o / part_ml and the
  // CTA that finishes last (counters) merges them.  No split when part_o is null.
  int sms = 0;
  float* part_o = nullptr;    // [slots][128][64] F32, one slot per (split CTA, query tile)
  float* part_ml = nullptr;   // [slots][128][2] F32: reference max (log2 domain), row sum
  int* counters = nullptr;    // [tail units][2] (at least part_slots ints), zero between launches
  int part_slots = 0;
  // Filled in by launch_flash (kernel-side view of the plan).
  int n_full = 0;
  int splits = 1;
  int items = 0;  // persistent layout: work items (units, split pieces or (segment, head, pair))
  // K'/V exchange of a sharded global block: key rows outside this rank's own rows
  // [own_begin, own_end) arrive from the peers.  peer_flags[r] = epoch << 32 |
  // complete << 31 | end once peer r's rows up to window row `end` are in place
  // (complete: all of them); the ranks' slices are contiguous in rank order.  The
  // producer starts at the first key tile of its own rows and waits (bounded) only
  // for the rows of the next tile it loads.  nullptr: nothing to wait for.
  const unsigned long long* peer_flags = nullptr;
  int epoch = 0;
  int nranks = 0;
  int rank = 0;
  int own_begin = 0;
  int own_end = 0;
};
// Launch plan of the attention kernel, computed on the host alone: launch_flash runs
// it, va_flash_plan reports it.
struct FlashPlan {
  int form = 0, poly = 0;  // the variant the launch runs (poly + 8 * form)
  int unit_rows = 0;       // query rows of one unit before any key split (128 or 256)
  int per_sm = 1;          // CTAs of this form resident per SM
  bool tile1 = false, persistent = false, w20 = false;
  int grid_x = 0, grid_y = 0, grid_z = 0;
};
// The shapes every TMA box of a launch needs (q, key window, segments).
bool flash_shapes_valid(const FlashArgs& fa);
// Resolves the default variant, validates it, and fills fa.n_full / splits / items
// and the plan for `sms` multiprocessors; one_tile_per_sm = resident CTAs of the
// one-tile form; split_ok = the caller gave a split workspace of fa.part_slots.
cudaError_t flash_plan(FlashArgs& fa, int sms, int one_tile_per_sm, bool split_ok, FlashPlan* plan);

// Value of an exchange flag (see FlashArgs::peer_flags).
inline unsigned long long peer_flag_value(int epoch, bool complete, int64_t end) {
  return (static_cast<unsigned long long>(static_cast<unsigned>(epoch)) << 32) |
         (complete ? (1ull << 31) : 0ull) | static_cast<unsigned long long>(end & 0x7fffffff);
}
// Slots a context provides for the split tail: rem < sms units, at most 4 key
// ranges each, two query tiles per CTA.
inline int flash_part_slots(int sms) { return 2 * 4 * sms; }

// Stream memory write (driver entry point cuStreamWriteValue32, no -lcuda needed):
// `value` lands at `addr` (this GPU's or a mapped peer's memory) once the stream's
// earlier work is done, behind a memory fence.  False when unavailable or refused.
bool stream_write_u32(cudaStream_t st, int* addr, uint32_t value);
// The same for a 64-bit value (cuStreamWriteValue64).
bool stream_write_u64(cudaStream_t st, unsigned long long* addr, unsigned long long value);

// Tensor-map encoding through the driver entry point (no -lcuda needed).
bool encode_tma_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                        uint32_t box_inner, uint32_t box_outer);
// Same for F32 [outer][inner] (used by TMA stores of F32 output tiles).
bool encode_tma_2d_f32(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                       uint32_t box_inner, uint32_t box_outer);
bool encode_tma_3d_bf16(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                        uint32_t b0, uint32_t b1, uint32_t b2);
// F32 [d2][d1][d0] with explicit byte strides of dims 1 and 2 (rows of a view and
// views), SWIZZLE_128B (box b0 * 4 bytes = 128).
bool encode_tma_3d_f32_strided(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1,
                               uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                               uint32_t b0, uint32_t b1, uint32_t b2);

// Launchers return cudaSuccess or the launch error; kernels report device-side
// failures through *err (see DevError in va_ptx.cuh).
cudaError_t launch_qkv_gemm(const __nv_bfloat16* x, const __nv_bfloat16* w_qkv_t, int rows,
                            int embed, const QkvEpilogueArgs& epi, int* err, cudaStream_t st);
// General form: out[m, n] from a[m, k] and w_t[n, k]; epi.embed is the output width n.
cudaError_t launch_proj_gemm(const __nv_bfloat16* a, const __nv_bfloat16* w_t, int m, int n, int k,
                             const ProjEpilogueArgs& epi, int* err, cudaStream_t st);
cudaError_t launch_flash(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v,
                         const FlashArgs& fa, int* err, cudaStream_t st);

// LN1 (optional) + F32 -> bf16 cast of token rows: x[rows,E] -> y[rows,E].
cudaError_t launch_ln_cast(const float* x, const float* g, const float* b, float eps, int rows,
                           int embed, __nv_bfloat16* y, cudaStream_t st);
// Op::Attention operand preparation: [H,n,64] F32 -> optional LN -> optional RoPE ->
// token-major bf16 [n][H*64].
cudaError_t launch_prep_heads(const float* x, int heads, int n, const float* g, const float* b,
                              float eps, const int2* pos, const float2* rope_cs, int rope_pairing,
                              __nv_bfloat16* y, cudaStream_t st, bool out_f16 = false);
// Camera-token slots (backbone.rs:746-768): token 0 of view 0 <- cam[0:E],
// token 0 of every later view <- cam[E:2E].
cudaError_t launch_camera_inject(float* tokens, const float* cam, int views, int tokens_per_view,
                                 int embed, cudaStream_t st, bool first_is_reference = true);
// View permutation: dst view i <- src view order[i] (order on the device).
cudaError_t launch_capture(const float* x, const float* local_x, const float* g, const float* b,
                           float eps, int views, int n, int n_special, int E, int cat, float* feat,
                           float* cam, cudaStream_t st);
cudaError_t launch_bounded_wait_selftest(unsigned long long limit_ns, int* err, cudaStream_t st);
cudaError_t launch_permute_views(const float* src, float* dst, const int* order, int views,
                                 int64_t view_elems, cudaStream_t st);

// ---- token input side (patch projection, CLS/register/position assembly) ----
// NCHW F32 images [views][3][H][W] -> bf16 patch rows [views*gh*gw][kp], feature
// index c*patch*patch + ky*patch + kx (the OIHW filter's flattening), zero past 3*patch^2.
cudaError_t launch_patchify(const float* img, int views, int height, int width, int patch, int kp,
                            __nv_bfloat16* rows, cudaStream_t st);
// Band form for patch 14 (kp 640) and width % 4 == 0 with the band in shared memory:
// also writes every view's special rows (as launch_token_specials).
constexpr int kPatchBandMaxSmem = 200 * 1024;
bool patchify_band_fits(int width, int patch, int kp);
cudaError_t launch_patchify_band(const float* img, int views, int height, int width, int patch, int kp,
                                 __nv_bfloat16* rows, const float* cls, const float* pos,
                                 const float* registers, int n_register, int n_tok, int embed,
                                 float* tokens, cudaStream_t st);
// Bicubic (a = -0.75) resampling of the learned [grid*grid + 1][E] table to
// [1 + gh*gw][E], CLS row copied.
cudaError_t launch_pos_interp(const float* pos_embed, int grid, int embed, int gh, int gw,
                              float interp_offset, float* out, cudaStream_t st);
// Special rows of every view: row 0 = cls + pos[0], rows 1..n_register = registers.
cudaError_t launch_token_specials(const float* cls, const float* pos, const float* registers,
                                  int n_register, int views, int n_tok, int embed, float* out,
                                  cudaStream_t st);
// Patch projection GEMM: a = patch rows [rows][k] bf16, w_t = filter [E][k] bf16.
cudaError_t launch_patch_gemm(const __nv_bfloat16* a, const __nv_bfloat16* w_t, int k,
                              const PatchEpilogueArgs& epi, int* err, cudaStream_t st);

// ---- GGUF model files (va_gguf.cu) ----
// One tensor of an open file after the checks of the reference's tensor_f32.
struct GgufTensorRef {
  int dtype;            // 0 F32, 1 F16, 8 Q8_0
  int ndims;
  int64_t shape[8];     // outer -> inner (stored dims reversed); 1 past ndims
  int64_t numel;
  const uint8_t* data;  // the stored bytes inside the file mapping
  size_t bytes;
};
// VA_OK, VA_ERR_NOT_FOUND (absent), or the failing check's code; message in gguf_message().
int gguf_tensor_ref(const va_gguf* g, const char* name, GgufTensorRef* out);
const char* gguf_message();
// Stored bytes (device copy, 256-byte aligned) -> F32 or bf16.  Not transposed:
// dst[r*ld + c] = value(r*cols + c); transposed: dst[c*ld + r] = value(r*cols + c).
cudaError_t launch_gguf_convert(const uint8_t* src, int dtype, int64_t rows, int64_t cols, int64_t ld,
                                bool transpose, bool out_bf16, void* dst, cudaStream_t st);
// Streams tensors to the device through two pinned staging buffers on its own
// stream: the host copy of one tensor overlaps the upload and conversion of the last.
class GgufStager {
 public:
  ~GgufStager();
  cudaError_t convert(const GgufTensorRef& t, int64_t rows, int64_t cols, int64_t ld, bool transpose,
                      bool out_bf16, void* dst);
  cudaError_t zero(void* dst, size_t bytes);  // cudaMemsetAsync on the staging stream
  cudaError_t finish();  // waits for every conversion issued so far
  size_t uploaded = 0;   // stored bytes sent to the device
 private:
  cudaError_t reserve(size_t bytes);
  void release();
  cudaStream_t stream_ = nullptr;
  cudaEvent_t ev_[2] = {};
  uint8_t* pinned_[2] = {};
  uint8_t* raw_[2] = {};
  bool used_[2] = {};
  size_t cap_ = 0;
  int slot_ = 0;
};

}  // namespace va
