// C-ABI layer: context, weight ownership, workspace, position tables and the
// per-call launch sequence of the attention path.
//
// Per attention sub-block call (vit_block.rs:772-992), one rank:
//   ln_cast  (LN1 when fused, F32 -> bf16)       [rows, E]
//   qkv_gemm (K1: UMMA + bias/QK-norm/RoPE epi)  -> Q, K, V bf16 token-major [rows, E]
//   [all-gather of K/V slices over NCCL when the window is sharded across GPUs]
//   flash    (K2: fused attention)               -> O bf16 [rows, E]
//   proj     (K3: UMMA + bias/ls1/residual epi)  -> F32 [rows, E]
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/vestra_attn.h"
#include "va_comm.h"
#include "va_internal.h"
#include "va_ptx.cuh"

using va::DevError;

namespace {

struct LayerWeights {
  bool loaded = false;
  bool in_arena = false;               // buffers carved from the model-file arena (not freed one by one)
  __nv_bfloat16* w_qkv_t = nullptr;   // [3E][E]
  __nv_bfloat16* w_proj_t = nullptr;  // [E][E]
  float* qkv_b = nullptr;             // [3E]
  float* proj_b = nullptr;            // [E]
  float* ls1 = nullptr;               // [E] or null
  float* norm1_w = nullptr;           // [E] or null
  float* norm1_b = nullptr;
  float* qn_g = nullptr;              // [64] or null (absent tensor)
  float* qn_b = nullptr;
  float* kn_g = nullptr;
  float* kn_b = nullptr;
  // Bound on |q.k| * scale * log2(e) after this layer's QK-norm (qk_bound_log2);
  // infinite without QK-norm tensors.
  float qk_bound = INFINITY;
};

constexpr int kMaxHostChunks = 32;
constexpr int kPhases = 5;
constexpr int kArenaWindows = 6;  // three key/value window pairs

// MLP sub-block of one block (vit_block.rs:131-236): LN2, fc1 (+GELU), fc2 (+ls2).
struct MlpWeights {
  bool loaded = false;
  bool in_arena = false;
  int hidden = 0;
  float* norm2_w = nullptr;           // [E]
  float* norm2_b = nullptr;
  __nv_bfloat16* w_fc1_t = nullptr;   // [hidden][E]
  float* fc1_b = nullptr;             // [hidden]
  __nv_bfloat16* w_fc2_t = nullptr;   // [E][hidden]
  float* fc2_b = nullptr;             // [E]
  float* ls2 = nullptr;               // [E] or null
};

// Patch projection and token assembly (patch_embed.rs:33-36, pos_embed.rs:23-39).
struct PatchEmbedWeights {
  bool loaded = false;
  bool in_arena = false;  // w_t, bias, cls, pos, regs from the model-file arena (rows is always its own)
  int patch = 0;
  int kp = 0;          // 3*patch^2 rounded up to the GEMM's 64-wide K slab
  int grid = 0;        // side of the learned position grid
  int n_register = 0;
  float offset = 0.1f; // interpolation offset (interp_offset)
  __nv_bfloat16* w_t = nullptr;   // [E][kp] filter rows, zero past 3*patch^2
  float* bias = nullptr;          // [E]
  float* cls = nullptr;           // [E]
  float* pos = nullptr;           // [(grid*grid + 1)][E]
  float* regs = nullptr;          // [n_register][E] or null
  __nv_bfloat16* rows = nullptr;  // own patch-row buffer [cap][kp] when kp > E (else the LN1 buffer)
};

struct PosKey {
  int64_t rows = -1;
  int gh = 0, gw = 0, views = 0, global = 0, n_special = 0;
  bool operator==(const PosKey& o) const {
    return rows == o.rows && gh == o.gh && gw == o.gw && views == o.views && global == o.global &&
           n_special == o.n_special;
  }
};

}  // namespace

struct va_ctx {
  va_config cfg{};
  int device = 0;
  std::vector<LayerWeights> layers;
  std::vector<MlpWeights> mlps;
  __nv_bfloat16* hbuf = nullptr;  // MLP hidden activations [cap][hidden_cap] bf16
  int hidden_cap = 0;
  // multi-layer device route (va_backbone_device)
  float* local_snap = nullptr;    // [cap][E] tokens after the last local block before a global one
  float* vit_norm_w = nullptr;    // [E] final-norm affine of the captures
  float* vit_norm_b = nullptr;
  bool vit_norm_in_arena = false;
  // QK-normalised layers whose score bound allows it run the softmax with a fixed
  // exponent offset (no row max); VA_SOFTMAX_FIXED_OFFSET=0 forces the row max.
  bool fixed_softmax = true;
  // Weights read from a model file (va_load_model_gguf) live in a few large chunks
  // carved in order, so a load makes a handful of allocations instead of one per tensor.
  std::vector<void*> weight_chunks;
  size_t chunk_used = 0, chunk_cap = 0;
  int64_t cap = 0;  // workspace rows
  __nv_bfloat16* x = nullptr;  // [cap][E] LN1 output, bf16
  __nv_bfloat16* q = nullptr;  // [cap][E] this rank's queries, token-major
  __nv_bfloat16* k = nullptr;  // [cap][E] key window (all ranks' slices after the gather)
  __nv_bfloat16* v = nullptr;  // [cap][E]
  // One allocation holds three key/value window pairs and the exchange flags, so
  // one IPC handle maps all of it into the peer processes.  Pair 0 (k, v) is this
  // rank's own (single-GPU and local calls); the direct K'/V exchange alternates
  // between pairs 1 and 2 call by call, so a peer only ever writes the pair this
  // rank read two sharded calls ago and never one another call is using.
  void* kv_arena = nullptr;
  size_t win_bytes = 0;
  int* xflags = nullptr;       // [kMaxRanks] exchange flags, written by the peers
  __nv_bfloat16* o = nullptr;  // [cap][E] attention output, token-major
  float* in_f32 = nullptr;     // host-path staging [cap][E]
  float* out_f32 = nullptr;
  int2* pos = nullptr;         // [cap] explicit tables (va_run_attention)
  // Closed-form position tables by shape, least recently used evicted: a layer loop
  // alternating local and global blocks finds both tables resident and launches
  // without uploads or synchronisation.
  struct PosEntry {
    PosKey key;
    int2* dev = nullptr;
    int64_t cap = 0;
    uint64_t used = 0;
  };
  PosEntry pos_cache[4];
  uint64_t pos_clock = 0;
  float2* rope_cs = nullptr;   // [rope_npos][16] (Op::Attention operand preparation)
  float2* rope_cs_t = nullptr; // the same values i-major, [16][rope_npos] (QKV epilogue)
  int rope_npos = 0;
  int* err = nullptr;          // device error word
  cudaStream_t stream = nullptr;
  // host path (va_attention_host): copy streams and per-chunk events
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t ev_in[kMaxHostChunks] = {};
  cudaEvent_t ev_out[kMaxHostChunks] = {};
  // Pipelined host batches alternate two staging pairs (in_f32/out_f32 and these):
  // copy-out chunk j of pair p done, and the last QKV chunk has read pair p's input.
  float* in_f32_alt = nullptr;
  float* out_f32_alt = nullptr;
  cudaEvent_t ev_d2h[2][kMaxHostChunks] = {};
  cudaEvent_t ev_in_free[2] = {};
  int sms = 148;
  // phase profile (va_set_phase_profile): events between the launches of the last
  // device-path call: ln | qkv+qk_norm_rope | all-gather | core | proj
  bool phase_profile = false;
  bool phase_valid = false;
  cudaEvent_t ph_ev[kPhases + 1] = {};
  // split-key tail of the attention kernel: partial rows and arrival counters
  float* part_o = nullptr;     // [2*sms][128][64]
  float* part_ml = nullptr;    // [2*sms][128][2]
  int* part_count = nullptr;   // [2*sms]
  // Op::Attention scratch (grown on demand)
  __nv_bfloat16* op_buf = nullptr;  // q|k|v bf16 [3][H*n*64]
  size_t op_cap = 0;
  int2* op_pos = nullptr;
  size_t op_pos_cap = 0;
  va::Comm* comm = nullptr;    // set by va_comm_init (multi-GPU global blocks)
  // direct K'/V exchange over NVLink (va_comm_init; else NCCL all-gather)
  bool p2p = false;
  // Copy-engine form of it: the QKV epilogue writes only this rank's rows; one
  // stream per peer copies them into that peer's window and then raises this
  // rank's flag there (a stream memory write, no SM involved); the attention kernel
  // waits on the flags itself.  Else the epilogue stores to the peers (SM stores)
  // and a barrier kernel follows.
  bool ce = false;
  cudaStream_t ce_st[va::kMaxPeers] = {};
  cudaEvent_t ce_ev[va::kMaxPeers] = {};
  cudaEvent_t ev_qkv = nullptr;
  // 64-bit exchange flags (FlashArgs::peer_flags), written by the peers; 128 bytes
  // into the flag area of the arena.
  unsigned long long* xflags64 = nullptr;
  // Copy-engine push plan: rows are pushed in chunks per peer (each followed by its
  // flag; push_chunks, or 0: one per 16 MB per peer, at most 4), on one stream per
  // peer, or with push_stagger on one stream peer after peer, the peer that reads
  // this rank's rows first (rank - 1) first.  VA_PUSH_CHUNKS / VA_PUSH_ORDER.
  int push_chunks = 0;
  bool push_stagger = true;
  // Copy engines carry a call's K'/V only from ce_min_peer_bytes per peer up: below
  // that the QKV epilogue's peer stores win (measured on 8 B200s: 4 MB per peer,
  // 0.160 vs 0.218 ms per S=12 sub-block; 16 MB at 2 GPUs: 0.327 vs 0.288 ms).
  // VA_KV_EXCHANGE=ce forces copy engines for every size.
  int64_t ce_min_peer_bytes = int64_t(12) << 20;
  int last_xchg = 0;  // path of the last sharded call (va_last_exchange)
  // With the phase profile on: per-peer push times of the last sharded call
  // (events around each peer's copies).
  cudaEvent_t ce_t0[va::kMaxPeers] = {};
  cudaEvent_t ce_t1[va::kMaxPeers] = {};
  int xchg_peers = 0;
  int64_t xchg_bytes = 0;
  int epoch = 0;
  void* peer_arena[va::kMaxRanks] = {};
  // token input side (va_load_patch_embed)
  PatchEmbedWeights pe;
  // Interpolated position tables [(1 + gh*gw)][E] by patch grid, least recently
  // used evicted (PosEmbedCache, pos_embed.rs:183-222, on the device).
  struct PosTable {
    int gh = 0, gw = 0;
    float* dev = nullptr;
    uint64_t used = 0;
  };
  PosTable pe_cache[4];
  uint64_t pe_clock = 0;
  std::string last_error;
};

namespace {

int fail(va_ctx* c, int code, const std::string& msg) {
  if (c) c->last_error = msg;
  return code;
}

int cuda_fail(va_ctx* c, cudaError_t e, const char* what) {
  return fail(c, VA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define VA_CUDA(ctx, call)                                   \
  do {                                                       \
    cudaError_t e_ = (call);                                 \
    if (e_ != cudaSuccess) return cuda_fail(ctx, e_, #call); \
  } while (0)

template <class T>
cudaError_t dmalloc(T** p, size_t count) {
  return cudaMalloc(reinterpret_cast<void**>(p), std::max<size_t>(count, 1) * sizeof(T));
}

template <class T>
void dfree(T*& p) {
  if (p) cudaFree(p);
  p = nullptr;
}

uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) return static_cast<uint16_t>((u >> 16) | ((u & 0xffff) ? 0x40 : 0));
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

// [in, out] F32 -> transposed [out][in] bf16 (K-major B operand).
std::vector<uint16_t> transpose_to_bf16(const float* w, int in, int out) {
  std::vector<uint16_t> t(static_cast<size_t>(in) * out);
  for (int i = 0; i < in; ++i)
    for (int o = 0; o < out; ++o) t[static_cast<size_t>(o) * in + i] = f32_to_bf16_rne(w[static_cast<size_t>(i) * out + o]);
  return t;
}

int upload_vec(va_ctx* c, float** dst, const float* src, size_t n) {
  if (!src) {
    *dst = nullptr;
    return VA_OK;
  }
  VA_CUDA(c, dmalloc(dst, n));
  VA_CUDA(c, cudaMemcpy(*dst, src, n * sizeof(float), cudaMemcpyHostToDevice));
  return VA_OK;
}

// Frees a device buffer the set owns, or forgets one carved from the weight arena.
template <class T>
void release(T*& p, bool in_arena) {
  if (in_arena)
    p = nullptr;
  else
    dfree(p);
}

void free_layer(LayerWeights& l) {
  const bool a = l.in_arena;
  release(l.w_qkv_t, a);
  release(l.w_proj_t, a);
  release(l.qkv_b, a);
  release(l.proj_b, a);
  release(l.ls1, a);
  release(l.norm1_w, a);
  release(l.norm1_b, a);
  release(l.qn_g, a);
  release(l.qn_b, a);
  release(l.kn_g, a);
  release(l.kn_b, a);
  l.qk_bound = INFINITY;
  l.in_arena = false;
  l.loaded = false;
}

// Bound on |q.k| * scale * log2(e) for a layer with QK-norm.  Each q (or k) head row
// is gamma * xhat + beta with xhat a LayerNorm output, |xhat| <= sqrt(d), so |q| <=
// max|gamma| sqrt(d) + |beta|; the 2D RoPE rotates pairs of components (norm kept).
// 2 % covers the bf16 rounding of q and k.  Non-finite weights give infinity.
float qk_bound_log2(const float* qg, const float* qb, const float* kg, const float* kb, int d) {
  auto row_bound = [d](const float* g, const float* b) {
    double mg = 0.0, sb = 0.0;
    for (int i = 0; i < d; ++i) {
      mg = std::max(mg, std::fabs(static_cast<double>(g[i])));
      sb += static_cast<double>(b[i]) * b[i];
    }
    return mg * std::sqrt(static_cast<double>(d)) + std::sqrt(sb);
  };
  const double bound = row_bound(qg, qb) * row_bound(kg, kb) / std::sqrt(static_cast<double>(d)) *
                       1.4426950408889634 * 1.02;
  return std::isfinite(bound) ? static_cast<float>(bound) : INFINITY;
}

// Largest bound for which the attention kernel may use exponents relative to 0
// (FlashArgs::fixed_offset): every 2^x then lies in [2^-64, 2^64].
constexpr float kFixedOffsetMaxBound = 64.0f;

void free_mlp(MlpWeights& m) {
  const bool a = m.in_arena;
  release(m.norm2_w, a);
  release(m.norm2_b, a);
  release(m.w_fc1_t, a);
  release(m.fc1_b, a);
  release(m.w_fc2_t, a);
  release(m.fc2_b, a);
  release(m.ls2, a);
  m.in_arena = false;
  m.loaded = false;
}

void free_vit_norm(va_ctx* c) {
  release(c->vit_norm_w, c->vit_norm_in_arena);
  release(c->vit_norm_b, c->vit_norm_in_arena);
  c->vit_norm_in_arena = false;
}

void free_patch_embed(va_ctx* c) {
  PatchEmbedWeights& p = c->pe;
  const bool a = p.in_arena;
  release(p.w_t, a);
  release(p.bias, a);
  release(p.cls, a);
  release(p.pos, a);
  release(p.regs, a);
  dfree(p.rows);
  p.in_arena = false;
  p.loaded = false;
  for (auto& e : c->pe_cache) {
    dfree(e.dev);
    e = va_ctx::PosTable{};
  }
}

// The interpolated position table of patch grid (gh, gw), built on `st` on first use.
int ensure_pos_table(va_ctx* c, int gh, int gw, cudaStream_t st, const float** out) {
  va_ctx::PosTable* hit = nullptr;
  for (auto& e : c->pe_cache)
    if (e.dev && e.gh == gh && e.gw == gw) hit = &e;
  if (!hit) {
    hit = &c->pe_cache[0];
    for (auto& e : c->pe_cache)
      if (e.used < hit->used) hit = &e;
    dfree(hit->dev);  // cudaFree waits for work still reading the evicted table
    *hit = va_ctx::PosTable{};
    VA_CUDA(c, dmalloc(&hit->dev, static_cast<size_t>(1 + gh * gw) * c->cfg.embed_dim));
    VA_CUDA(c, va::launch_pos_interp(c->pe.pos, c->pe.grid, c->cfg.embed_dim, gh, gw, c->pe.offset,
                                     hit->dev, st));
    // Built once per grid; finishing it here lets later calls on any stream read it.
    VA_CUDA(c, cudaStreamSynchronize(st));
    hit->gh = gh;
    hit->gw = gw;
  }
  hit->used = ++c->pe_clock;
  *out = hit->dev;
  return VA_OK;
}

bool layer_use_qknorm(const va_ctx* c, int layer) {
  return c->cfg.qknorm_start >= 0 && layer >= c->cfg.qknorm_start && c->layers[layer].qn_g != nullptr;
}
bool layer_use_rope(const va_ctx* c, int layer) {
  return c->cfg.rope_start >= 0 && layer >= c->cfg.rope_start;
}

// cos/sin table of pos * base^(-2i/32), i < 16, for pos in [0, npos).  Double on
// the host, rounded to F32, like the CPU restatement.
int ensure_rope_table(va_ctx* c, int npos) {
  if (npos <= c->rope_npos) return VA_OK;
  const int n = std::max(npos, 64);
  std::vector<float2> t(static_cast<size_t>(n) * 16);
  for (int p = 0; p < n; ++p)
    for (int i = 0; i < 16; ++i) {
      const double ang = p * std::pow(static_cast<double>(c->cfg.rope_freq), -(2.0 * i) / 32.0);
      t[static_cast<size_t>(p) * 16 + i] = make_float2(static_cast<float>(std::cos(ang)),
                                                      static_cast<float>(std::sin(ang)));
    }
  std::vector<float2> tt(t.size());
  for (int p = 0; p < n; ++p)
    for (int i = 0; i < 16; ++i) tt[static_cast<size_t>(i) * n + p] = t[static_cast<size_t>(p) * 16 + i];
  dfree(c->rope_cs);
  dfree(c->rope_cs_t);
  VA_CUDA(c, dmalloc(&c->rope_cs, t.size()));
  VA_CUDA(c, cudaMemcpy(c->rope_cs, t.data(), t.size() * sizeof(float2), cudaMemcpyHostToDevice));
  VA_CUDA(c, dmalloc(&c->rope_cs_t, tt.size()));
  VA_CUDA(c, cudaMemcpy(c->rope_cs_t, tt.data(), tt.size() * sizeof(float2), cudaMemcpyHostToDevice));
  c->rope_npos = n;
  return VA_OK;
}

// Closed-form position table (vit_block.rs:841-881) of one window shape, from the
// context's cache; *out receives the device table.
int ensure_positions(va_ctx* c, int64_t rows, int gh, int gw, int views, int global,
                     const int2** out) {
  const int n_special = 1 + c->cfg.num_register;
  PosKey key{rows, gh, gw, views, global, n_special};
  for (auto& e : c->pos_cache)
    if (e.dev && e.key == key) {
      e.used = ++c->pos_clock;
      *out = e.dev;
      return VA_OK;
    }
  const int64_t per_view = n_special + static_cast<int64_t>(gh) * gw;
  if (views <= 0 || per_view * views != rows)
    return fail(c, VA_ERR_INVALID, "rows must equal view_count * (1 + num_register + gh*gw)");
  std::vector<int2> p(static_cast<size_t>(rows), make_int2(0, 0));
  int maxp = 1;
  for (int v = 0; v < views; ++v)
    for (int64_t lt = n_special; lt < per_view; ++lt) {
      const int64_t t = v * per_view + lt;
      if (global) {
        p[t] = make_int2(1, 1);
      } else {
        const int64_t q = lt - n_special;
        p[t] = make_int2(static_cast<int>(q / gw + 1), static_cast<int>(q % gw + 1));
        maxp = std::max(maxp, std::max(p[t].x, p[t].y));
      }
    }
  va_ctx::PosEntry* slot = &c->pos_cache[0];
  for (auto& e : c->pos_cache)
    if (!e.dev || e.used < slot->used) slot = &e;
  // The evicted table (or a smaller rope table) may still be read by queued kernels.
  if (slot->dev || maxp + 1 > c->rope_npos) VA_CUDA(c, cudaDeviceSynchronize());
  int rc = ensure_rope_table(c, maxp + 1);
  if (rc) return rc;
  if (slot->cap < rows) {
    dfree(slot->dev);
    slot->cap = 0;
    VA_CUDA(c, dmalloc(&slot->dev, static_cast<size_t>(rows)));
    slot->cap = rows;
  }
  VA_CUDA(c, cudaMemcpy(slot->dev, p.data(), p.size() * sizeof(int2), cudaMemcpyHostToDevice));
  slot->key = key;
  slot->used = ++c->pos_clock;
  *out = slot->dev;
  return VA_OK;
}

// Explicit F32 position table (AttentionExecutor seam) -> c->pos.
int upload_positions(va_ctx* c, const float* pos_yx, int64_t rows, int2* dst) {
  std::vector<int2> p(static_cast<size_t>(rows));
  int maxp = 0;
  for (int64_t t = 0; t < rows; ++t) {
    const long long y = std::llround(pos_yx[2 * t]), x = std::llround(pos_yx[2 * t + 1]);
    if (y < 0 || x < 0 || y > 65535 || x > 65535)
      return fail(c, VA_ERR_INVALID, "RoPE positions must be integers in [0, 65535]");
    p[t] = make_int2(static_cast<int>(y), static_cast<int>(x));
    maxp = std::max(maxp, static_cast<int>(std::max(y, x)));
  }
  VA_CUDA(c, cudaDeviceSynchronize());  // the old table may still be in use
  int rc = ensure_rope_table(c, maxp + 1);
  if (rc) return rc;
  VA_CUDA(c, cudaMemcpy(dst, p.data(), p.size() * sizeof(int2), cudaMemcpyHostToDevice));
  return VA_OK;
}

int check_layer(va_ctx* c, int layer) {
  if (layer < 0 || layer >= static_cast<int>(c->layers.size()))
    return fail(c, VA_ERR_INVALID, "layer index out of range");
  if (!c->layers[layer].loaded) return fail(c, VA_ERR_STATE, "layer weights not loaded");
  return VA_OK;
}

// One rank's share of an attention sub-block.  The key window holds window_rows
// tokens; this rank owns rows [row_offset, row_offset + rows) of it (single GPU:
// row_offset 0, rows == window_rows).
struct BranchSpec {
  const float* in;        // F32 [rows, E]: LN1 output, or raw tokens when apply_ln1
  bool apply_ln1;
  float* out;             // F32 [rows, E]
  const float* residual;  // F32 [rows, E] added in the epilogue, or nullptr
  int64_t rows;
  int64_t row_offset;
  int64_t window_rows;
  const int2* pos;        // positions of the window (nullptr: no RoPE)
  int seg_len;            // 0: global attention over the window; > 0: per-view segments
  bool gather;            // all-gather K/V slices of every rank before the attention
  __nv_bfloat16* kwin;    // key / value window buffers of this call
  __nv_bfloat16* vwin;
  int npeer;              // direct exchange: peers whose windows receive this slice
  __nv_bfloat16* peer_k[va::kMaxPeers];
  __nv_bfloat16* peer_v[va::kMaxPeers];
  bool ce = false;        // copy-engine exchange (see va_ctx::ce)
  int epoch = 0;
  unsigned long long* peer_flag[va::kMaxPeers] = {};  // this rank's flag in each peer's flag array
  int peer_rank[va::kMaxPeers] = {};
};

// In-place all-gather of this rank's K'/V slices into the window buffers.
int gather_kv(va_ctx* c, const __nv_bfloat16* k_slice, const __nv_bfloat16* v_slice, int64_t rows,
              cudaStream_t st) {
  if (!c->comm) return fail(c, VA_ERR_STATE, "no communicator (va_comm_init)");
  const size_t per_rank = static_cast<size_t>(rows) * c->cfg.embed_dim;
  if (k_slice != c->k + per_rank * va::comm_rank(c->comm) ||
      v_slice != c->v + per_rank * va::comm_rank(c->comm))
    return fail(c, VA_ERR_INVALID, "sharded slices must be rank-ordered and equal");
  std::string err;
  if (!va::comm_allgather_inplace2(c->comm, c->k, c->v, per_rank, st, &err))
    return fail(c, VA_ERR_NCCL, err);
  return VA_OK;
}

void close_peers(va_ctx* c) {
  for (int r = 0; r < va::kMaxRanks; ++r) {
    if (c->peer_arena[r]) cudaIpcCloseMemHandle(c->peer_arena[r]);
    c->peer_arena[r] = nullptr;
  }
  c->p2p = false;
  c->ce = false;
}

// Maps every peer's kv_arena into this process (CUDA IPC) for the direct K'/V
// exchange.  Every rank's outcome is all-gathered and the direct exchange is used
// only when every rank mapped every peer; otherwise the NCCL all-gather stays in
// use.  VA_KV_EXCHANGE=nccl forces the all-gather.  The flags are cleared before
// the first collective, so no peer can have written one yet.
int setup_peers(va_ctx* c) {
  close_peers(c);
  c->epoch = 0;
  VA_CUDA(c, cudaMemset(c->xflags, 0, 256));
  VA_CUDA(c, cudaDeviceSynchronize());
  const int nranks = va::comm_size(c->comm), rank = va::comm_rank(c->comm);
  if (nranks < 2 || nranks > va::kMaxRanks) return VA_OK;
  const char* env = std::getenv("VA_KV_EXCHANGE");
  const bool forced_nccl = env && std::string(env) == "nccl";
  // "sm": direct exchange by the QKV epilogue's stores (no copy-engine push).
  const bool forced_sm = env && std::string(env) == "sm";
  struct Slot {
    cudaIpcMemHandle_t h;
    int ok;
    int pad;
    unsigned long long win_bytes;  // every rank's arena must have the same layout
    int pad2[12];
  };
  static_assert(sizeof(Slot) == 128, "slot size");
  Slot mine{};
  mine.ok = 0;
  mine.win_bytes = c->win_bytes;
  if (!forced_nccl) {
    mine.ok = cudaIpcGetMemHandle(&mine.h, c->kv_arena) == cudaSuccess;
    if (!mine.ok) cudaGetLastError();
  }
  Slot* dbuf = nullptr;
  VA_CUDA(c, dmalloc(&dbuf, static_cast<size_t>(nranks) + 1));
  std::vector<Slot> all(nranks);
  std::string err;
  int rc = VA_OK;
  cudaError_t e = cudaMemcpy(dbuf + nranks, &mine, sizeof(Slot), cudaMemcpyHostToDevice);
  if (e == cudaSuccess && !va::comm_allgather_bytes(c->comm, dbuf + nranks, dbuf, sizeof(Slot), c->stream, &err))
    rc = fail(c, VA_ERR_NCCL, err);
  if (e == cudaSuccess && rc == VA_OK) e = cudaStreamSynchronize(c->stream);
  if (e == cudaSuccess && rc == VA_OK)
    e = cudaMemcpy(all.data(), dbuf, sizeof(Slot) * nranks, cudaMemcpyDeviceToHost);
  int opened = rc == VA_OK && e == cudaSuccess;
  for (int r = 0; opened && r < nranks; ++r) {
    if (!all[r].ok || all[r].win_bytes != c->win_bytes) opened = 0;
    if (!opened || r == rank) continue;
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, all[r].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      opened = 0;
    } else {
      c->peer_arena[r] = p;
    }
  }
  // The copy-engine push needs stream memory writes into a peer's memory: write 0
  // (the flags' value before any call) into this rank's slot of every peer.
  int ce_ok = 0;
  if (opened && !forced_sm) {
    ce_ok = 1;
    for (int r = 0; ce_ok && r < nranks; ++r) {
      if (r == rank) continue;
      auto* slot = reinterpret_cast<unsigned long long*>(static_cast<char*>(c->peer_arena[r]) +
                                                         kArenaWindows * c->win_bytes + 128) + rank;
      ce_ok = va::stream_write_u64(c->stream, slot, 0ull) ? 1 : 0;
    }
    if (cudaStreamSynchronize(c->stream) != cudaSuccess) {
      cudaGetLastError();
      ce_ok = 0;
    }
  }
  // Second round: the direct exchange only if every rank mapped every peer, its
  // copy-engine form only if every rank's stream writes worked.
  if (rc == VA_OK) {
    std::vector<Slot> flags(nranks);
    Slot f{};
    f.ok = opened | (ce_ok << 1);
    e = cudaMemcpy(dbuf + nranks, &f, sizeof(Slot), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && !va::comm_allgather_bytes(c->comm, dbuf + nranks, dbuf, sizeof(Slot), c->stream, &err))
      rc = fail(c, VA_ERR_NCCL, err);
    if (e == cudaSuccess && rc == VA_OK) e = cudaStreamSynchronize(c->stream);
    if (e == cudaSuccess && rc == VA_OK)
      e = cudaMemcpy(flags.data(), dbuf, sizeof(Slot) * nranks, cudaMemcpyDeviceToHost);
    bool all_ok = e == cudaSuccess && rc == VA_OK, all_ce = all_ok;
    for (int r = 0; all_ok && r < nranks; ++r) all_ok = (flags[r].ok & 1) != 0;
    for (int r = 0; all_ce && r < nranks; ++r) all_ce = (flags[r].ok & 2) != 0;
    c->p2p = all_ok;
    c->ce = all_ok && all_ce;
  }
  cudaFree(dbuf);
  if (!c->p2p) close_peers(c);
  if (rc == VA_OK && e != cudaSuccess) rc = cuda_fail(c, e, "peer window exchange");
  return rc;
}

int segments_for(va_ctx* c, int64_t rows, int view_count, int global, int* seg_len) {
  if (view_count <= 0 || rows % view_count != 0)
    return fail(c, VA_ERR_INVALID, "rows must be a multiple of view_count");
  *seg_len = global ? 0 : static_cast<int>(rows / view_count);
  return VA_OK;
}

// Hands the context's partial-result workspace to a flash launch (split tail).
void set_split_workspace(const va_ctx* c, va::FlashArgs* fa) {
  fa->sms = c->sms;
  fa->part_o = c->part_o;
  fa->part_ml = c->part_ml;
  fa->counters = c->part_count;
  fa->part_slots = va::flash_part_slots(c->sms);
}

int validate_branch(va_ctx* c, int layer, const BranchSpec& b) {
  const LayerWeights& w = c->layers[layer];
  if (!b.in || !b.out || !b.kwin || !b.vwin) return fail(c, VA_ERR_INVALID, "missing buffer");
  if (b.rows <= 0 || b.window_rows > c->cap || b.row_offset + b.rows > b.window_rows)
    return fail(c, VA_ERR_INVALID, "rows exceed the context's max_rows");
  if (b.window_rows > 0x7fffffff / 64) return fail(c, VA_ERR_INVALID, "rows too large");
  if (b.apply_ln1 && !w.norm1_w) return fail(c, VA_ERR_STATE, "norm1 weights not loaded");
  if (b.seg_len > 0 && (b.rows % b.seg_len != 0 || b.row_offset % b.seg_len != 0))
    return fail(c, VA_ERR_INVALID, "a rank's rows must hold whole views in local blocks");
  if (b.seg_len == 0 && !b.gather && b.rows != b.window_rows)
    return fail(c, VA_ERR_INVALID, "global attention over a sharded window needs the communicator");
  return VA_OK;
}

// Projection stage for rows [r0, r1) of this rank's slice: LN1 / bf16 cast, then
// the QKV GEMM with its bias + QK-norm + RoPE epilogue; Q' goes to c->q, K' and V
// to the rank's rows of the key window.
int stage_qkv(va_ctx* c, int layer, const BranchSpec& b, int64_t r0, int64_t r1, cudaStream_t st,
              cudaEvent_t between = nullptr) {
  const LayerWeights& w = c->layers[layer];
  const int E = c->cfg.embed_dim;
  const int n = static_cast<int>(r1 - r0);
  VA_CUDA(c, va::launch_ln_cast(b.in + r0 * E, b.apply_ln1 ? w.norm1_w : nullptr, w.norm1_b,
                                c->cfg.ln_eps, n, E, c->x + r0 * E, st));
  if (between) VA_CUDA(c, cudaEventRecord(between, st));
  va::QkvEpilogueArgs qa{};
  qa.bias = w.qkv_b;
  const bool qk = layer_use_qknorm(c, layer);
  qa.q_g = qk ? w.qn_g : nullptr;
  qa.q_b = qk ? w.qn_b : nullptr;
  qa.k_g = qk ? w.kn_g : nullptr;
  qa.k_b = qk ? w.kn_b : nullptr;
  qa.qk_eps = c->cfg.qk_norm_eps;
  qa.pos = b.pos ? b.pos + b.row_offset + r0 : nullptr;
  qa.rope_cs = c->rope_cs_t;
  qa.rope_npos = c->rope_npos;
  qa.rope_pairing = c->cfg.rope_pairing;
  qa.q_out = c->q + r0 * E;
  qa.k_out = b.kwin + (b.row_offset + r0) * E;
  qa.v_out = b.vwin + (b.row_offset + r0) * E;
  qa.npeer = b.ce ? 0 : b.npeer;
  for (int p = 0; p < qa.npeer; ++p) {
    qa.peer_k[p] = b.peer_k[p] + (b.row_offset + r0) * E;
    qa.peer_v[p] = b.peer_v[p] + (b.row_offset + r0) * E;
  }
  qa.rows = n;
  qa.embed = E;
  // V (and so P) stay bf16: measured faster on B200 than an f16 P formed with
  // packed ex2.f16x2 (584 vs 511 TFLOP/s for the S=12 window).
  qa.v_f16 = 0;
  VA_CUDA(c, va::launch_qkv_gemm(c->x + r0 * E, w.w_qkv_t, n, E, qa, c->err, st));
  return VA_OK;
}

// Attention stage for this rank's queries [q0, q1): fused flash attention against
// the key window (global) or the queries' own views (local; the range then holds
// whole views), then the output projection with its bias/ls1/residual epilogue.
int stage_attn(va_ctx* c, int layer, const BranchSpec& b, int64_t q0, int64_t q1, cudaStream_t st,
               cudaEvent_t between = nullptr) {
  const LayerWeights& w = c->layers[layer];
  const int E = c->cfg.embed_dim;
  const int n = static_cast<int>(q1 - q0);
  va::FlashArgs fa{};
  fa.q_count = n;
  fa.seg_len = b.seg_len;
  fa.heads = c->cfg.num_heads;
  fa.scale_log2 = static_cast<float>(1.0 / std::sqrt(64.0) * 1.4426950408889634);
  fa.out_mode = 0;
  fa.o_tok = c->o + q0 * E;
  fa.embed = E;
  fa.v_f16 = 0;
  fa.fixed_offset = c->fixed_softmax && layer_use_qknorm(c, layer) &&
                    c->layers[layer].qk_bound <= kFixedOffsetMaxBound;
  const __nv_bfloat16* kk = b.kwin;
  const __nv_bfloat16* vv = b.vwin;
  if (b.seg_len > 0) {
    // Local blocks: every key a query needs lives in its own view.
    kk = b.kwin + (b.row_offset + q0) * E;
    vv = b.vwin + (b.row_offset + q0) * E;
    fa.q_offset = 0;
    fa.kv_rows = n;
  } else {
    fa.q_offset = static_cast<int>(b.row_offset + q0);
    fa.kv_rows = static_cast<int>(b.window_rows);
    if (b.npeer > 0) {
      fa.peer_flags = c->xflags64;
      fa.epoch = b.epoch;
      fa.nranks = va::comm_size(c->comm);
      fa.rank = va::comm_rank(c->comm);
      fa.own_begin = static_cast<int>(b.row_offset);
      fa.own_end = static_cast<int>(b.row_offset + b.rows);
    }
  }
  set_split_workspace(c, &fa);
  VA_CUDA(c, va::launch_flash(c->q + q0 * E, kk, vv, fa, c->err, st));
  if (between) VA_CUDA(c, cudaEventRecord(between, st));
  va::ProjEpilogueArgs pa{};
  pa.bias = w.proj_b;
  pa.ls1 = w.ls1;
  pa.residual = b.residual ? b.residual + q0 * E : nullptr;
  pa.out = b.out + q0 * E;
  pa.rows = n;
  pa.embed = E;
  VA_CUDA(c, va::launch_proj_gemm(c->o + q0 * E, w.w_proj_t, n, E, E, pa, c->err, st));
  return VA_OK;
}

// The device launch sequence of one attention sub-block (see the file header).
// Direct K'/V exchange of one sharded call: picks the call's window pair (1 or 2,
// alternating) and every peer's copy of it, and fills the barrier arguments.
// Returns false when the call uses no direct exchange.
bool prepare_exchange(va_ctx* c, BranchSpec* b) {
  if (!b->gather || !c->p2p) return false;
  const int nranks = va::comm_size(c->comm), rank = va::comm_rank(c->comm);
  const int set = 1 + ((++c->epoch) & 1);
  const size_t win = c->win_bytes;
  char* own = static_cast<char*>(c->kv_arena);
  b->kwin = reinterpret_cast<__nv_bfloat16*>(own + (2 * set) * win);
  b->vwin = reinterpret_cast<__nv_bfloat16*>(own + (2 * set + 1) * win);
  b->npeer = 0;
  for (int r = 0; r < nranks; ++r) {
    if (r == rank) continue;
    char* pa = static_cast<char*>(c->peer_arena[r]);
    b->peer_k[b->npeer] = reinterpret_cast<__nv_bfloat16*>(pa + (2 * set) * win);
    b->peer_v[b->npeer] = reinterpret_cast<__nv_bfloat16*>(pa + (2 * set + 1) * win);
    b->peer_flag[b->npeer] = reinterpret_cast<unsigned long long*>(pa + kArenaWindows * win + 128) + rank;
    b->peer_rank[b->npeer] = r;
    ++b->npeer;
  }
  const int64_t peer_bytes = b->rows * c->cfg.embed_dim * 2 * static_cast<int64_t>(sizeof(__nv_bfloat16));
  b->ce = c->ce && peer_bytes >= c->ce_min_peer_bytes;
  b->epoch = c->epoch;
  c->last_xchg = b->ce ? 3 : 2;
  return true;
}

// The copy-engine push of this rank's K'/V rows (after its QKV on `st`): per peer,
// the rows in push_chunks chunks (K then V), each chunk followed by the peer's flag
// (epoch, rows delivered so far, complete after the last chunk).  One copy stream
// per peer, or with push_stagger one stream that serves the peers in the order they
// read this rank's rows (rank - 1 first).
int push_rows(va_ctx* c, const BranchSpec& b, cudaStream_t st) {
  const int E = c->cfg.embed_dim;
  const int nranks = va::comm_size(c->comm), rank = va::comm_rank(c->comm);
  VA_CUDA(c, cudaEventRecord(c->ev_qkv, st));
  // Chunks: the VA_PUSH_CHUNKS setting, else one per 16 MB sent to a peer (each copy
  // costs ~10 us of its own, so small slices go in one piece), at most 4.
  const int64_t peer_bytes = b.rows * E * 2 * static_cast<int64_t>(sizeof(__nv_bfloat16));
  const int64_t want = c->push_chunks > 0 ? c->push_chunks : std::min<int64_t>(4, (peer_bytes + (16 << 20) - 1) >> 24);
  const int chunks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, b.rows / 64)));
  const bool prof = c->phase_profile;
  for (int k = 1; k < nranks; ++k) {
    const int dst = (rank - k + nranks) % nranks;
    const int p = dst < rank ? dst : dst - 1;  // peer index (peers in rank order)
    cudaStream_t cs = c->ce_st[b.ce && c->push_stagger ? 0 : p];
    if (!c->push_stagger || k == 1) VA_CUDA(c, cudaStreamWaitEvent(cs, c->ev_qkv, 0));
    if (prof) VA_CUDA(c, cudaEventRecord(c->ce_t0[p], cs));
    for (int ch = 0; ch < chunks; ++ch) {
      const int64_t r0 = b.row_offset + b.rows * ch / chunks, r1 = b.row_offset + b.rows * (ch + 1) / chunks;
      const size_t off = static_cast<size_t>(r0) * E;
      const size_t bytes = static_cast<size_t>(r1 - r0) * E * sizeof(__nv_bfloat16);
      VA_CUDA(c, cudaMemcpyAsync(b.peer_k[p] + off, b.kwin + off, bytes, cudaMemcpyDeviceToDevice, cs));
      VA_CUDA(c, cudaMemcpyAsync(b.peer_v[p] + off, b.vwin + off, bytes, cudaMemcpyDeviceToDevice, cs));
      if (!va::stream_write_u64(cs, b.peer_flag[p], va::peer_flag_value(b.epoch, ch + 1 == chunks, r1)))
        return fail(c, VA_ERR_CUDA, "stream flag write to a peer failed");
    }
    if (prof) VA_CUDA(c, cudaEventRecord(c->ce_t1[p], cs));
  }
  for (int p = 0; p < b.npeer; ++p)
    if (!c->push_stagger || p == 0) VA_CUDA(c, cudaEventRecord(c->ce_ev[p], c->ce_st[p]));
  c->xchg_peers = prof ? b.npeer : 0;
  c->xchg_bytes = b.rows * E * 2 * static_cast<int64_t>(sizeof(__nv_bfloat16));
  return VA_OK;
}

// `st` waits for every copy stream of the call (the copies read this rank's rows,
// which the call after next overwrites).
int join_push(va_ctx* c, const BranchSpec& b, cudaStream_t st) {
  for (int p = 0; b.ce && p < b.npeer; ++p)
    if (!c->push_stagger || p == 0) VA_CUDA(c, cudaStreamWaitEvent(st, c->ce_ev[p], 0));
  return VA_OK;
}

// The exchange step between the projection and the attention of a sharded call:
// the copy-engine push, the flags after the epilogue's peer stores, or the NCCL
// all-gather.
int exchange_step(va_ctx* c, const BranchSpec& b, bool direct, cudaStream_t st) {
  if (direct && b.ce) {
    return push_rows(c, b, st);
  } else if (direct) {
    va::PeerFlagArgs pf{};
    pf.npeer = b.npeer;
    for (int p = 0; p < b.npeer; ++p) pf.peer_flag[p] = b.peer_flag[p];
    pf.value = va::peer_flag_value(b.epoch, true, b.row_offset + b.rows);
    VA_CUDA(c, va::launch_peer_flags(pf, st));
  } else if (b.gather) {
    c->last_xchg = 1;
    const int E = c->cfg.embed_dim;
    return gather_kv(c, c->k + b.row_offset * E, c->v + b.row_offset * E, b.rows, st);
  }
  return VA_OK;
}

// The device launch sequence of one attention sub-block (see the file header).
int run_branch(va_ctx* c, int layer, const BranchSpec& b_in, cudaStream_t st) {
  int rc = validate_branch(c, layer, b_in);
  if (rc) return rc;
  BranchSpec b = b_in;
  const bool direct = prepare_exchange(c, &b);
  // With the phase profile on, an event goes between every two launches; the ln
  // and qkv phases are split inside stage_qkv's two launches by mark(1).
  const bool prof = c->phase_profile;
  auto mark = [&](int i) { return prof ? cudaEventRecord(c->ph_ev[i], st) : cudaSuccess; };
  c->phase_valid = false;
  c->xchg_peers = 0;
  VA_CUDA(c, mark(0));
  if ((rc = stage_qkv(c, layer, b, 0, b.rows, st, prof ? c->ph_ev[1] : nullptr))) return rc;
  VA_CUDA(c, mark(2));
  if ((rc = exchange_step(c, b, direct, st))) return rc;
  VA_CUDA(c, mark(3));
  if ((rc = stage_attn(c, layer, b, 0, b.rows, st, prof ? c->ph_ev[4] : nullptr))) return rc;
  if ((rc = join_push(c, b, st))) return rc;
  VA_CUDA(c, mark(5));
  c->phase_valid = prof;
  return VA_OK;
}

int host_call(va_ctx* c, int layer, struct BranchSpec b, int view_count, const float* ln1, float* out);

int read_device_error(va_ctx* c) {
  int h = 0;
  VA_CUDA(c, cudaMemcpy(&h, c->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (h != 0) {
    cudaMemset(c->err, 0, sizeof(int));
    // An aborted split-tail CTA may have left an arrival counter behind.
    cudaMemset(c->part_count, 0, static_cast<size_t>(va::flash_part_slots(c->sms)) * sizeof(int));
    char buf[128];
    std::snprintf(buf, sizeof(buf), "device error word %d (a bounded wait timed out)", h);
    return fail(c, VA_ERR_DEVICE, buf);
  }
  return VA_OK;
}

}  // namespace

extern "C" {

const char* va_version(void) { return "vestra_attn 0.1 sm_100a"; }

void va_default_config(va_config* cfg) {
  if (!cfg) return;
  cfg->embed_dim = 768;
  cfg->num_heads = 12;
  cfg->head_dim = 64;
  cfg->depth = 12;
  cfg->num_register = 0;
  cfg->rope_start = 4;
  cfg->qknorm_start = 4;
  cfg->rope_freq = 100.0f;
  cfg->ln_eps = 1e-6f;
  cfg->qk_norm_eps = 1e-5f;
  cfg->rope_pairing = 0;
  cfg->max_rows = 12 * 866;
}

int va_create(const va_config* cfg, int device, va_ctx** out) {
  if (!cfg || !out) return VA_ERR_INVALID;
  *out = nullptr;
  if (cfg->head_dim != 64 || cfg->embed_dim != cfg->num_heads * 64 || cfg->embed_dim % 256 != 0 ||
      cfg->depth <= 0 || cfg->max_rows <= 0 || cfg->num_register < 0 ||
      (cfg->rope_pairing != 0 && cfg->rope_pairing != 1))
    return VA_ERR_INVALID;
  va_ctx* c = new (std::nothrow) va_ctx();
  if (!c) return VA_ERR_INVALID;
  c->cfg = *cfg;
  c->device = device;
  c->layers.resize(cfg->depth);
  c->mlps.resize(cfg->depth);
  c->cap = cfg->max_rows;
  auto bail = [&](cudaError_t e) {
    va_destroy(c);
    (void)e;
    return VA_ERR_CUDA;
  };
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return bail(e);
  const size_t E = cfg->embed_dim;
  const size_t n = static_cast<size_t>(c->cap) * E;
  if ((e = dmalloc(&c->x, n)) != cudaSuccess) return bail(e);
  if ((e = dmalloc(&c->q, n)) != cudaSuccess) return bail(e);
  {
    const size_t win = n * sizeof(__nv_bfloat16);
    if ((e = cudaMalloc(&c->kv_arena, kArenaWindows * win + 256)) != cudaSuccess) return bail(e);
    char* a = static_cast<char*>(c->kv_arena);
    c->win_bytes = win;
    c->k = reinterpret_cast<__nv_bfloat16*>(a);
    c->v = reinterpret_cast<__nv_bfloat16*>(a + win);
    c->xflags = reinterpret_cast<int*>(a + kArenaWindows * win);
    c->xflags64 = reinterpret_cast<unsigned long long*>(a + kArenaWindows * win + 128);
    if ((e = cudaMemset(c->xflags, 0, 256)) != cudaSuccess) return bail(e);
  }
  if ((e = dmalloc(&c->o, n)) != cudaSuccess) return bail(e);
  if ((e = dmalloc(&c->in_f32, n)) != cudaSuccess) return bail(e);
  if ((e = dmalloc(&c->out_f32, n)) != cudaSuccess) return bail(e);
  if ((e = dmalloc(&c->pos, static_cast<size_t>(c->cap))) != cudaSuccess) return bail(e);
  if ((e = dmalloc(&c->err, 1)) != cudaSuccess) return bail(e);
  if ((e = cudaMemset(c->err, 0, sizeof(int))) != cudaSuccess) return bail(e);
  {
    const char* fx = std::getenv("VA_SOFTMAX_FIXED_OFFSET");
    c->fixed_softmax = !(fx && fx[0] == '0');
  }
  if ((e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking)) != cudaSuccess) return bail(e);
  if ((e = cudaStreamCreateWithFlags(&c->h2d, cudaStreamNonBlocking)) != cudaSuccess) return bail(e);
  if ((e = cudaStreamCreateWithFlags(&c->d2h, cudaStreamNonBlocking)) != cudaSuccess) return bail(e);
  for (int i = 0; i < kMaxHostChunks; ++i) {
    if ((e = cudaEventCreateWithFlags(&c->ev_in[i], cudaEventDisableTiming)) != cudaSuccess) return bail(e);
    if ((e = cudaEventCreateWithFlags(&c->ev_out[i], cudaEventDisableTiming)) != cudaSuccess) return bail(e);
    for (int p = 0; p < 2; ++p)
      if ((e = cudaEventCreateWithFlags(&c->ev_d2h[p][i], cudaEventDisableTiming)) != cudaSuccess) return bail(e);
  }
  for (int p = 0; p < 2; ++p)
    if ((e = cudaEventCreateWithFlags(&c->ev_in_free[p], cudaEventDisableTiming)) != cudaSuccess) return bail(e);
  if ((e = cudaDeviceGetAttribute(&c->sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess)
    return bail(e);
  for (int i = 0; i <= kPhases; ++i)
    if ((e = cudaEventCreate(&c->ph_ev[i])) != cudaSuccess) return bail(e);
  for (int p = 0; p < va::kMaxPeers; ++p) {
    if ((e = cudaStreamCreateWithFlags(&c->ce_st[p], cudaStreamNonBlocking)) != cudaSuccess) return bail(e);
    if ((e = cudaEventCreateWithFlags(&c->ce_ev[p], cudaEventDisableTiming)) != cudaSuccess) return bail(e);
  }
  if ((e = cudaEventCreateWithFlags(&c->ev_qkv, cudaEventDisableTiming)) != cudaSuccess) return bail(e);
  for (int p = 0; p < va::kMaxPeers; ++p) {
    if ((e = cudaEventCreate(&c->ce_t0[p])) != cudaSuccess) return bail(e);
    if ((e = cudaEventCreate(&c->ce_t1[p])) != cudaSuccess) return bail(e);
  }
  {
    const char* pc = std::getenv("VA_PUSH_CHUNKS");
    if (pc && std::atoi(pc) >= 1 && std::atoi(pc) <= 16) c->push_chunks = std::atoi(pc);
    const char* po = std::getenv("VA_PUSH_ORDER");
    if (po) c->push_stagger = std::string(po) != "parallel";
    const char* xe = std::getenv("VA_KV_EXCHANGE");
    if (xe && std::string(xe) == "ce") c->ce_min_peer_bytes = 0;
  }
  {
    const size_t slots = static_cast<size_t>(va::flash_part_slots(c->sms));
    if ((e = dmalloc(&c->part_o, slots * 128 * 64)) != cudaSuccess) return bail(e);
    if ((e = dmalloc(&c->part_ml, slots * 128 * 2)) != cudaSuccess) return bail(e);
    if ((e = dmalloc(&c->part_count, slots)) != cudaSuccess) return bail(e);
    if ((e = cudaMemset(c->part_count, 0, slots * sizeof(int))) != cudaSuccess) return bail(e);
  }
  if (ensure_rope_table(c, 128) != VA_OK) return bail(cudaErrorMemoryAllocation);
  *out = c;
  return VA_OK;
}

void va_destroy(va_ctx* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  if (c->h2d) cudaStreamSynchronize(c->h2d);
  if (c->d2h) cudaStreamSynchronize(c->d2h);
  for (auto& l : c->layers) free_layer(l);
  for (auto& m : c->mlps) free_mlp(m);
  free_patch_embed(c);
  free_vit_norm(c);
  for (void* chunk : c->weight_chunks) cudaFree(chunk);
  c->weight_chunks.clear();
  dfree(c->hbuf);
  dfree(c->local_snap);
  dfree(c->x);
  dfree(c->q);
  close_peers(c);
  if (c->kv_arena) cudaFree(c->kv_arena);
  c->kv_arena = nullptr;
  dfree(c->o);
  dfree(c->in_f32);
  dfree(c->out_f32);
  dfree(c->in_f32_alt);
  dfree(c->out_f32_alt);
  dfree(c->pos);
  for (auto& e : c->pos_cache) dfree(e.dev);
  dfree(c->rope_cs);
  dfree(c->rope_cs_t);
  dfree(c->err);
  dfree(c->op_buf);
  dfree(c->op_pos);
  dfree(c->part_o);
  dfree(c->part_ml);
  dfree(c->part_count);
  if (c->comm) va::comm_destroy(c->comm, false);
  if (c->stream) cudaStreamDestroy(c->stream);
  if (c->h2d) cudaStreamDestroy(c->h2d);
  if (c->d2h) cudaStreamDestroy(c->d2h);
  for (int i = 0; i < kMaxHostChunks; ++i) {
    if (c->ev_in[i]) cudaEventDestroy(c->ev_in[i]);
    if (c->ev_out[i]) cudaEventDestroy(c->ev_out[i]);
    for (int p = 0; p < 2; ++p)
      if (c->ev_d2h[p][i]) cudaEventDestroy(c->ev_d2h[p][i]);
  }
  for (int p = 0; p < 2; ++p)
    if (c->ev_in_free[p]) cudaEventDestroy(c->ev_in_free[p]);
  for (int i = 0; i <= kPhases; ++i)
    if (c->ph_ev[i]) cudaEventDestroy(c->ph_ev[i]);
  for (int p = 0; p < va::kMaxPeers; ++p) {
    if (c->ce_st[p]) {
      cudaStreamSynchronize(c->ce_st[p]);
      cudaStreamDestroy(c->ce_st[p]);
    }
    if (c->ce_ev[p]) cudaEventDestroy(c->ce_ev[p]);
  }
  if (c->ev_qkv) cudaEventDestroy(c->ev_qkv);
  for (int p = 0; p < va::kMaxPeers; ++p) {
    if (c->ce_t0[p]) cudaEventDestroy(c->ce_t0[p]);
    if (c->ce_t1[p]) cudaEventDestroy(c->ce_t1[p]);
  }
  delete c;
}

const char* va_last_error(const va_ctx* c) { return c ? c->last_error.c_str() : "null context"; }

int va_load_layer(va_ctx* c, int layer, const float* norm1_w, const float* norm1_b,
                  const float* qkv_w, const float* qkv_b, const float* qnorm_w,
                  const float* qnorm_b, const float* knorm_w, const float* knorm_b,
                  const float* proj_w, const float* proj_b, const float* ls1) {
  if (!c) return VA_ERR_INVALID;
  if (layer < 0 || layer >= c->cfg.depth) return fail(c, VA_ERR_INVALID, "layer index out of range");
  if (!qkv_w || !qkv_b || !proj_w || !proj_b)
    return fail(c, VA_ERR_INVALID, "qkv and proj weights are required");
  if ((qnorm_w == nullptr) != (knorm_w == nullptr) || (qnorm_w && (!qnorm_b || !knorm_b)))
    return fail(c, VA_ERR_INVALID, "q-norm and k-norm tensors must be given together");
  if ((norm1_w == nullptr) != (norm1_b == nullptr))
    return fail(c, VA_ERR_INVALID, "norm1 weight and bias must be given together");
  VA_CUDA(c, cudaSetDevice(c->device));
  LayerWeights& l = c->layers[layer];
  free_layer(l);
  const int E = c->cfg.embed_dim;
  std::vector<uint16_t> wq = transpose_to_bf16(qkv_w, E, 3 * E);
  std::vector<uint16_t> wp = transpose_to_bf16(proj_w, E, E);
  VA_CUDA(c, dmalloc(&l.w_qkv_t, wq.size()));
  VA_CUDA(c, cudaMemcpy(l.w_qkv_t, wq.data(), wq.size() * 2, cudaMemcpyHostToDevice));
  VA_CUDA(c, dmalloc(&l.w_proj_t, wp.size()));
  VA_CUDA(c, cudaMemcpy(l.w_proj_t, wp.data(), wp.size() * 2, cudaMemcpyHostToDevice));
  int rc;
  if ((rc = upload_vec(c, &l.qkv_b, qkv_b, 3 * E))) return rc;
  if ((rc = upload_vec(c, &l.proj_b, proj_b, E))) return rc;
  if ((rc = upload_vec(c, &l.ls1, ls1, E))) return rc;
  if ((rc = upload_vec(c, &l.norm1_w, norm1_w, E))) return rc;
  if ((rc = upload_vec(c, &l.norm1_b, norm1_b, E))) return rc;
  if ((rc = upload_vec(c, &l.qn_g, qnorm_w, 64))) return rc;
  if ((rc = upload_vec(c, &l.qn_b, qnorm_b, 64))) return rc;
  if ((rc = upload_vec(c, &l.kn_g, knorm_w, 64))) return rc;
  if ((rc = upload_vec(c, &l.kn_b, knorm_b, 64))) return rc;
  l.qk_bound = qnorm_w ? qk_bound_log2(qnorm_w, qnorm_b, knorm_w, knorm_b, 64) : INFINITY;
  l.loaded = true;
  return VA_OK;
}

int va_load_mlp(va_ctx* c, int layer, int mlp_hidden, const float* norm2_w, const float* norm2_b,
                const float* fc1_w, const float* fc1_b, const float* fc2_w, const float* fc2_b,
                const float* ls2) {
  if (!c) return VA_ERR_INVALID;
  if (layer < 0 || layer >= c->cfg.depth) return fail(c, VA_ERR_INVALID, "layer index out of range");
  if (!norm2_w || !norm2_b || !fc1_w || !fc1_b || !fc2_w || !fc2_b)
    return fail(c, VA_ERR_INVALID, "norm2, fc1 and fc2 tensors are required");
  if (mlp_hidden <= 0 || mlp_hidden % 256 != 0)
    return fail(c, VA_ERR_INVALID, "mlp_hidden must be a positive multiple of 256");
  VA_CUDA(c, cudaSetDevice(c->device));
  VA_CUDA(c, cudaDeviceSynchronize());  // earlier calls may still read the old weights / buffer
  MlpWeights& m = c->mlps[layer];
  free_mlp(m);
  const int E = c->cfg.embed_dim;
  if (mlp_hidden > c->hidden_cap) {
    dfree(c->hbuf);
    VA_CUDA(c, dmalloc(&c->hbuf, static_cast<size_t>(c->cap) * mlp_hidden));
    c->hidden_cap = mlp_hidden;
  }
  std::vector<uint16_t> w1 = transpose_to_bf16(fc1_w, E, mlp_hidden);
  std::vector<uint16_t> w2 = transpose_to_bf16(fc2_w, mlp_hidden, E);
  VA_CUDA(c, dmalloc(&m.w_fc1_t, w1.size()));
  VA_CUDA(c, cudaMemcpy(m.w_fc1_t, w1.data(), w1.size() * 2, cudaMemcpyHostToDevice));
  VA_CUDA(c, dmalloc(&m.w_fc2_t, w2.size()));
  VA_CUDA(c, cudaMemcpy(m.w_fc2_t, w2.data(), w2.size() * 2, cudaMemcpyHostToDevice));
  int rc;
  if ((rc = upload_vec(c, &m.norm2_w, norm2_w, E))) return rc;
  if ((rc = upload_vec(c, &m.norm2_b, norm2_b, E))) return rc;
  if ((rc = upload_vec(c, &m.fc1_b, fc1_b, mlp_hidden))) return rc;
  if ((rc = upload_vec(c, &m.fc2_b, fc2_b, E))) return rc;
  if ((rc = upload_vec(c, &m.ls2, ls2, E))) return rc;
  m.hidden = mlp_hidden;
  m.loaded = true;
  return VA_OK;
}

int va_layer_flags(const va_ctx* c, int layer, int* use_qknorm, int* use_rope) {
  if (!c || layer < 0 || layer >= c->cfg.depth) return VA_ERR_INVALID;
  if (use_qknorm) *use_qknorm = layer_use_qknorm(c, layer) ? 1 : 0;
  if (use_rope) *use_rope = layer_use_rope(c, layer) ? 1 : 0;
  return VA_OK;
}

int va_run_attention(va_ctx* c, int layer, const float* input, int64_t rows, int heads,
                     int head_dim, const float* positions_yx, float* out) {
  if (!c || !input || !out) return VA_ERR_INVALID;
  int rc = check_layer(c, layer);
  if (rc) return rc;
  if (heads != c->cfg.num_heads || head_dim != c->cfg.head_dim || rows <= 0)
    return fail(c, VA_ERR_INVALID, "heads/head_dim do not match the context");
  if (rows > c->cap) return fail(c, VA_ERR_INVALID, "rows exceed the context's max_rows");
  VA_CUDA(c, cudaSetDevice(c->device));
  const int2* pos = nullptr;
  if (positions_yx) {
    VA_CUDA(c, cudaStreamSynchronize(c->stream));  // c->pos may still be read by a previous call
    if ((rc = upload_positions(c, positions_yx, rows, c->pos))) return rc;
    pos = c->pos;
  }
  // The same chunked host pipeline as va_attention_host, so both seams compute
  // the same rows in the same launches (bitwise equal for equal positions).
  BranchSpec b{c->in_f32, false, c->out_f32, nullptr, rows, 0, rows, pos, 0, false, c->k, c->v, 0, {}, {}};
  if ((rc = validate_branch(c, layer, b))) return rc;
  return host_call(c, layer, b, 1, input, out);
}

}  // extern "C"

namespace {

// MLP sub-block in place on device tokens [rows][E] (vit_block.rs:1092-1129):
// LN2 + bf16 cast, fc1 GEMM with bias + exact GELU, fc2 GEMM with bias, ls2 and
// the residual add fused into its epilogue.
int run_mlp(va_ctx* c, int layer, float* tokens, int64_t rows, cudaStream_t st) {
  if (layer < 0 || layer >= c->cfg.depth || !c->mlps[layer].loaded)
    return fail(c, VA_ERR_STATE, "MLP weights not loaded (va_load_mlp)");
  if (rows <= 0 || rows > c->cap) return fail(c, VA_ERR_INVALID, "rows out of range");
  const MlpWeights& m = c->mlps[layer];
  const int E = c->cfg.embed_dim;
  const int n = static_cast<int>(rows);
  VA_CUDA(c, va::launch_ln_cast(tokens, m.norm2_w, m.norm2_b, c->cfg.ln_eps, n, E, c->x, st));
  va::Fc1EpilogueArgs fa{m.fc1_b, c->hbuf, n, m.hidden};
  VA_CUDA(c, va::launch_fc1_gemm(c->x, m.w_fc1_t, n, m.hidden, E, fa, c->err, st));
  va::ProjEpilogueArgs pa{};
  pa.bias = m.fc2_b;
  pa.ls1 = m.ls2;
  pa.residual = tokens;
  pa.out = tokens;
  pa.rows = n;
  pa.embed = E;
  VA_CUDA(c, va::launch_proj_gemm(c->hbuf, m.w_fc2_t, n, E, m.hidden, pa, c->err, st));
  return VA_OK;
}

// Checks a closed-form-position call and builds its BranchSpec.  window_rows = the
// whole view-major window (all ranks); local_rows = this rank's slice.
int make_branch(va_ctx* c, int layer, const float* in, bool apply_ln1, float* out,
                const float* residual, int64_t window_rows, int64_t local_rows, int64_t row_offset,
                int gh, int gw, int view_count, int global, bool sharded, BranchSpec* b) {
  int rc = check_layer(c, layer);
  if (rc) return rc;
  if (window_rows <= 0 || window_rows > c->cap) return fail(c, VA_ERR_INVALID, "rows out of range");
  int seg_len;
  if ((rc = segments_for(c, window_rows, view_count, global, &seg_len))) return rc;
  const int2* pos = nullptr;
  if (layer_use_rope(c, layer)) {
    if ((rc = ensure_positions(c, window_rows, gh, gw, view_count, global, &pos))) return rc;
  }
  *b = BranchSpec{in, apply_ln1, out, residual, local_rows, row_offset, window_rows, pos, seg_len,
                  sharded && global, c->k, c->v, 0, {}, {}};
  return validate_branch(c, layer, *b);
}

// Shared body of the closed-form-position device entry points.
int device_call(va_ctx* c, int layer, const float* in, bool apply_ln1, float* out,
                const float* residual, int64_t window_rows, int64_t local_rows, int64_t row_offset,
                int gh, int gw, int view_count, int global, bool sharded, cudaStream_t st) {
  BranchSpec b;
  int rc = make_branch(c, layer, in, apply_ln1, out, residual, window_rows, local_rows, row_offset,
                       gh, gw, view_count, global, sharded, &b);
  if (rc) return rc;
  return run_branch(c, layer, b, st);
}

// Row ranges [bounds[i], bounds[i+1]) of the host path's chunks.
using Bounds = std::vector<int64_t>;

Bounds split_rows(int64_t rows, int64_t step) {
  Bounds r;
  for (int64_t a = 0; a < rows; a += step) r.push_back(a);
  r.push_back(rows);
  return r;
}

// Chunking of the host path (va_attention_host).  Local blocks: groups of whole
// views, each copied in, projected, attended, projected out and copied back on its
// own, so the two copy directions overlap each other and the compute.  Global
// blocks: the input in up to 8 chunks of >= 1024 rows (their LN/QKV overlaps the
// later copies in), then the queries in chunks of about one wave of attention CTAs
// (sms / heads CTAs of 256 queries each), so the copy out of one chunk overlaps the
// attention of the next; no query can finish before the last key has arrived.
// (Smaller first chunks, split over key ranges, were measured slower on B200: 1.42
// and 1.48 ms against 1.39 ms per S=12 window, the extra launches and copies costing
// more than the earlier start of the copy-out.)
void plan_host_chunks(const va_ctx* c, const BranchSpec& b, int view_count, Bounds* in,
                      Bounds* out) {
  const int64_t rows = b.rows;
  if (b.seg_len > 0) {
    const int64_t views = rows / b.seg_len;
    const int64_t per = std::max<int64_t>(1, (views + 5) / 6);
    *in = split_rows(rows, per * b.seg_len);
    *out = *in;
    (void)view_count;
    return;
  }
  // At most 8 input chunks and at least 1024 rows each: a QKV launch of fewer rows
  // (under ~70 CTAs) leaves most SMs idle and, when sharded, starves the peer stores.
  const int64_t step_in = std::max<int64_t>(1024, ((rows + 7) / 8 + 127) / 128 * 128);
  *in = split_rows(rows, step_in);
  const int64_t pairs = (rows + 255) / 256;
  const int64_t per_wave = std::max<int64_t>(1, c->sms / std::max(1, c->cfg.num_heads));
  const int64_t n_out = std::min<int64_t>(kMaxHostChunks, (pairs + per_wave - 1) / per_wave);
  const int64_t per_chunk = (pairs + n_out - 1) / n_out;
  *out = split_rows(rows, per_chunk * 256);
}

// The host-buffer path of one sub-block call (this rank's rows), chunked so that
// the copies overlap the compute (see plan_host_chunks); for a sharded global
// block the K'/V exchange runs between the last projection chunk and the first
// attention chunk.
int host_call(va_ctx* c, int layer, BranchSpec b, int view_count, const float* ln1, float* out) {
  int rc = VA_OK;
  const bool direct = prepare_exchange(c, &b);
  Bounds in, outb;
  plan_host_chunks(c, b, view_count, &in, &outb);
  const int E = c->cfg.embed_dim;
  const size_t row_bytes = static_cast<size_t>(E) * sizeof(float);
  // Every stream is drained before returning, also on an error, so no copy still
  // reads or writes the caller's buffers afterwards.
  auto finish = [&](int code) {
    cudaStreamSynchronize(c->h2d);
    cudaStreamSynchronize(c->stream);
    cudaStreamSynchronize(c->d2h);
    return code;
  };
#define VA_HOST(call)                                                          \
  do {                                                                         \
    cudaError_t e_ = (call);                                                   \
    if (e_ != cudaSuccess) return finish(cuda_fail(c, e_, #call));             \
  } while (0)
  const int n_in = static_cast<int>(in.size()) - 1, n_out = static_cast<int>(outb.size()) - 1;
  for (int i = 0; i < n_in; ++i) {
    VA_HOST(cudaMemcpyAsync(c->in_f32 + in[i] * E, ln1 + in[i] * E, (in[i + 1] - in[i]) * row_bytes,
                            cudaMemcpyHostToDevice, c->h2d));
    VA_HOST(cudaEventRecord(c->ev_in[i], c->h2d));
  }
  for (int i = 0; i < n_in; ++i) {
    VA_HOST(cudaStreamWaitEvent(c->stream, c->ev_in[i], 0));
    if ((rc = stage_qkv(c, layer, b, in[i], in[i + 1], c->stream))) return finish(rc);
    if (b.seg_len > 0) {  // local: the chunk's views are complete
      if ((rc = stage_attn(c, layer, b, in[i], in[i + 1], c->stream))) return finish(rc);
      VA_HOST(cudaEventRecord(c->ev_out[i], c->stream));
    }
  }
  if (b.seg_len == 0) {
    if ((rc = exchange_step(c, b, direct, c->stream))) return finish(rc);
    for (int j = 0; j < n_out; ++j) {
      if ((rc = stage_attn(c, layer, b, outb[j], outb[j + 1], c->stream))) return finish(rc);
      VA_HOST(cudaEventRecord(c->ev_out[j], c->stream));
    }
    if ((rc = join_push(c, b, c->stream))) return finish(rc);
  }
  for (int j = 0; j < n_out; ++j) {
    VA_HOST(cudaStreamWaitEvent(c->d2h, c->ev_out[j], 0));
    VA_HOST(cudaMemcpyAsync(out + outb[j] * E, c->out_f32 + outb[j] * E,
                            (outb[j + 1] - outb[j]) * row_bytes, cudaMemcpyDeviceToHost, c->d2h));
  }
#undef VA_HOST
  VA_CUDA(c, cudaStreamSynchronize(c->d2h));
  finish(VA_OK);
  return read_device_error(c);
}

// host_call over independent steps of one shape (single GPU), pipelined.  Steps
// alternate two staging pairs (input F32, output F32), so step s's copy in only
// waits for step s-2's last QKV chunk and step s's projection of chunk j only for
// step s-2's copy out of that chunk: the copy in of one step, the compute of the
// next and the copy out of the one before run at once (both PCIe directions busy).
int host_batch(va_ctx* c, int layer, const BranchSpec& b0, int view_count, const float* const* ln1,
               float* const* out, int nsteps) {
  int rc = VA_OK;
  const int E = c->cfg.embed_dim;
  if (nsteps > 1 && !c->in_f32_alt) {
    VA_CUDA(c, dmalloc(&c->in_f32_alt, static_cast<size_t>(c->cap) * E));
    VA_CUDA(c, dmalloc(&c->out_f32_alt, static_cast<size_t>(c->cap) * E));
  }
  Bounds in, outb;
  plan_host_chunks(c, b0, view_count, &in, &outb);
  const size_t row_bytes = static_cast<size_t>(E) * sizeof(float);
  auto finish = [&](int code) {
    cudaStreamSynchronize(c->h2d);
    cudaStreamSynchronize(c->stream);
    cudaStreamSynchronize(c->d2h);
    return code;
  };
#define VA_HOST(call)                                                          \
  do {                                                                         \
    cudaError_t e_ = (call);                                                   \
    if (e_ != cudaSuccess) return finish(cuda_fail(c, e_, #call));             \
  } while (0)
  const int n_in = static_cast<int>(in.size()) - 1, n_out = static_cast<int>(outb.size()) - 1;
  for (int s = 0; s < nsteps; ++s) {
    const int p = s & 1;
    BranchSpec b = b0;
    b.in = p ? c->in_f32_alt : c->in_f32;
    b.out = p ? c->out_f32_alt : c->out_f32;
    float* in_buf = const_cast<float*>(b.in);
    if (s >= 2) VA_HOST(cudaStreamWaitEvent(c->h2d, c->ev_in_free[p], 0));
    for (int i = 0; i < n_in; ++i) {
      VA_HOST(cudaMemcpyAsync(in_buf + in[i] * E, ln1[s] + in[i] * E, (in[i + 1] - in[i]) * row_bytes,
                              cudaMemcpyHostToDevice, c->h2d));
      VA_HOST(cudaEventRecord(c->ev_in[i], c->h2d));
    }
    for (int i = 0; i < n_in; ++i) {
      VA_HOST(cudaStreamWaitEvent(c->stream, c->ev_in[i], 0));
      if ((rc = stage_qkv(c, layer, b, in[i], in[i + 1], c->stream))) return finish(rc);
      if (b.seg_len > 0) {  // local: the chunk's views are complete
        if (s >= 2) VA_HOST(cudaStreamWaitEvent(c->stream, c->ev_d2h[p][i], 0));
        if ((rc = stage_attn(c, layer, b, in[i], in[i + 1], c->stream))) return finish(rc);
        VA_HOST(cudaEventRecord(c->ev_out[i], c->stream));
      }
    }
    VA_HOST(cudaEventRecord(c->ev_in_free[p], c->stream));
    if (b.seg_len == 0) {
      for (int j = 0; j < n_out; ++j) {
        if (s >= 2) VA_HOST(cudaStreamWaitEvent(c->stream, c->ev_d2h[p][j], 0));
        if ((rc = stage_attn(c, layer, b, outb[j], outb[j + 1], c->stream))) return finish(rc);
        VA_HOST(cudaEventRecord(c->ev_out[j], c->stream));
      }
    }
    for (int j = 0; j < n_out; ++j) {
      VA_HOST(cudaStreamWaitEvent(c->d2h, c->ev_out[j], 0));
      VA_HOST(cudaMemcpyAsync(out[s] + outb[j] * E, b.out + outb[j] * E, (outb[j + 1] - outb[j]) * row_bytes,
                              cudaMemcpyDeviceToHost, c->d2h));
      VA_HOST(cudaEventRecord(c->ev_d2h[p][j], c->d2h));
    }
  }
#undef VA_HOST
  VA_CUDA(c, cudaStreamSynchronize(c->d2h));
  finish(VA_OK);
  return read_device_error(c);
}


}  // namespace

extern "C" {

int va_attention_host(va_ctx* c, int layer, const float* ln1, int64_t rows, int gh, int gw,
                      int view_count, int global, float* out) {
  if (!c || !ln1 || !out) return VA_ERR_INVALID;
  if (rows <= 0 || rows > c->cap) return fail(c, VA_ERR_INVALID, "rows out of range");
  VA_CUDA(c, cudaSetDevice(c->device));
  BranchSpec b;
  int rc = make_branch(c, layer, c->in_f32, false, c->out_f32, nullptr, rows, rows, 0, gh, gw,
                       view_count, global, false, &b);
  if (rc) return rc;
  return host_call(c, layer, b, view_count, ln1, out);
}

int va_attention_host_batch(va_ctx* c, int layer, const float* const* ln1, float* const* out, int nsteps,
                            int64_t rows, int gh, int gw, int view_count, int global) {
  if (!c || !ln1 || !out || nsteps < 0) return VA_ERR_INVALID;
  for (int s = 0; s < nsteps; ++s)
    if (!ln1[s] || !out[s]) return fail(c, VA_ERR_INVALID, "null step buffer");
  if (nsteps == 0) return VA_OK;
  if (rows <= 0 || rows > c->cap) return fail(c, VA_ERR_INVALID, "rows out of range");
  VA_CUDA(c, cudaSetDevice(c->device));
  BranchSpec b;
  int rc = make_branch(c, layer, c->in_f32, false, c->out_f32, nullptr, rows, rows, 0, gh, gw,
                       view_count, global, false, &b);
  if (rc) return rc;
  return host_batch(c, layer, b, view_count, ln1, out, nsteps);
}

int va_attention_host_sharded(va_ctx* c, int layer, const float* ln1_local, float* out_local,
                              int64_t local_rows, int gh, int gw, int view_count, int global) {
  if (!c || !ln1_local || !out_local) return VA_ERR_INVALID;
  if (local_rows <= 0 || local_rows > c->cap) return fail(c, VA_ERR_INVALID, "rows out of range");
  const int nranks = c->comm ? va::comm_size(c->comm) : 1;
  const int rank = c->comm ? va::comm_rank(c->comm) : 0;
  if (global && !c->comm) return fail(c, VA_ERR_STATE, "no communicator (va_comm_init)");
  VA_CUDA(c, cudaSetDevice(c->device));
  BranchSpec b;
  int rc = make_branch(c, layer, c->in_f32, false, c->out_f32, nullptr, local_rows * nranks,
                       local_rows, local_rows * rank, gh, gw, view_count, global, true, &b);
  if (rc) return rc;
  return host_call(c, layer, b, view_count, ln1_local, out_local);
}

int va_attention_device(va_ctx* c, int layer, const float* ln1_dev, float* out_dev, int64_t rows,
                        int gh, int gw, int view_count, int global, void* stream) {
  if (!c || !ln1_dev || !out_dev) return VA_ERR_INVALID;
  return device_call(c, layer, ln1_dev, false, out_dev, nullptr, rows, rows, 0, gh, gw, view_count,
                     global, false, static_cast<cudaStream_t>(stream));
}

int va_block_attention_device(va_ctx* c, int layer, float* tokens_dev, int64_t rows, int gh,
                              int gw, int view_count, int global, void* stream) {
  if (!c || !tokens_dev) return VA_ERR_INVALID;
  return device_call(c, layer, tokens_dev, true, tokens_dev, tokens_dev, rows, rows, 0, gh, gw,
                     view_count, global, false, static_cast<cudaStream_t>(stream));
}

int va_block_device(va_ctx* c, int layer, float* tokens_dev, int64_t rows, int gh, int gw,
                    int view_count, int global, void* stream) {
  if (!c || !tokens_dev) return VA_ERR_INVALID;
  if (layer < 0 || layer >= c->cfg.depth || !c->mlps[layer].loaded)
    return fail(c, VA_ERR_STATE, "MLP weights not loaded (va_load_mlp)");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = device_call(c, layer, tokens_dev, true, tokens_dev, tokens_dev, rows, rows, 0, gh, gw,
                       view_count, global, false, st);
  if (rc) return rc;
  return run_mlp(c, layer, tokens_dev, rows, st);
}

int va_load_vit_norm(va_ctx* c, const float* norm_w, const float* norm_b) {
  if (!c || !norm_w || !norm_b) return VA_ERR_INVALID;
  VA_CUDA(c, cudaSetDevice(c->device));
  VA_CUDA(c, cudaDeviceSynchronize());
  free_vit_norm(c);
  int rc;
  if ((rc = upload_vec(c, &c->vit_norm_w, norm_w, c->cfg.embed_dim))) return rc;
  return upload_vec(c, &c->vit_norm_b, norm_b, c->cfg.embed_dim);
}

int va_load_patch_embed(va_ctx* c, const float* weight_oihw, const float* bias,
                        const float* cls_token, const float* pos_embed, int64_t pos_rows,
                        const float* register_tokens, int num_register, int patch,
                        float interp_offset) {
  if (!c) return VA_ERR_INVALID;
  if (!weight_oihw || !bias || !cls_token || !pos_embed)
    return fail(c, VA_ERR_INVALID, "patch filter, bias, cls token and pos_embed are required");
  if (patch <= 0 || 3 * patch * patch > 4096) return fail(c, VA_ERR_INVALID, "patch size out of range");
  if (num_register != c->cfg.num_register || (num_register > 0 && !register_tokens))
    return fail(c, VA_ERR_INVALID, "num_register must match the context and come with its tokens");
  // infer_grid (pos_embed.rs:89-106): 1 CLS row + a square grid.
  const int64_t grid_rows = pos_rows - 1;
  int grid = static_cast<int>(std::llround(std::sqrt(static_cast<double>(std::max<int64_t>(grid_rows, 0)))));
  if (pos_rows < 2 || static_cast<int64_t>(grid) * grid != grid_rows)
    return fail(c, VA_ERR_INVALID, "pos_embed patch-row count is not a perfect square");
  VA_CUDA(c, cudaSetDevice(c->device));
  VA_CUDA(c, cudaDeviceSynchronize());
  free_patch_embed(c);
  const int E = c->cfg.embed_dim, features = 3 * patch * patch;
  const int kp = (features + 63) / 64 * 64;
  // OIHW [E][3][p][p] is already [E][features] K-major; pad K to kp with zeros.
  std::vector<uint16_t> w(static_cast<size_t>(E) * kp, 0);
  for (int o = 0; o < E; ++o)
    for (int i = 0; i < features; ++i)
      w[static_cast<size_t>(o) * kp + i] = f32_to_bf16_rne(weight_oihw[static_cast<size_t>(o) * features + i]);
  PatchEmbedWeights& p = c->pe;
  VA_CUDA(c, dmalloc(&p.w_t, w.size()));
  VA_CUDA(c, cudaMemcpy(p.w_t, w.data(), w.size() * 2, cudaMemcpyHostToDevice));
  int rc;
  if ((rc = upload_vec(c, &p.bias, bias, E))) return rc;
  if ((rc = upload_vec(c, &p.cls, cls_token, E))) return rc;
  if ((rc = upload_vec(c, &p.pos, pos_embed, static_cast<size_t>(pos_rows) * E))) return rc;
  if (num_register > 0 && (rc = upload_vec(c, &p.regs, register_tokens, static_cast<size_t>(num_register) * E)))
    return rc;
  if (kp > E) VA_CUDA(c, dmalloc(&p.rows, static_cast<size_t>(c->cap) * kp));
  p.patch = patch;
  p.kp = kp;
  p.grid = grid;
  p.n_register = num_register;
  p.offset = interp_offset;
  p.loaded = true;
  return VA_OK;
}

}  // extern "C"

namespace {

// One model file's tensors into the context's buffers (va_load_model_gguf).  The
// reference first builds host `Weights` (weights_from_gguf, engine.rs:110-126: a
// rank-2 tensor transposed, any other rank as stored) and the executors read
// linear weights from there as [in, out]; every conversion below writes what that
// content gives, directly in the device layout.
struct GgufLoad {
  va_ctx* c;
  const va_gguf* g;
  va::GgufStager st;

  // Next 256-byte-aligned piece of the weight arena, opening a new chunk of at
  // least 64 MiB when the current one is full.
  template <class T>
  int carve(T** p, size_t count) {
    const size_t bytes = (std::max<size_t>(count, 1) * sizeof(T) + 255) & ~static_cast<size_t>(255);
    if (c->weight_chunks.empty() || c->chunk_used + bytes > c->chunk_cap) {
      const size_t cap = std::max<size_t>(bytes, size_t(64) << 20);
      void* m = nullptr;
      VA_CUDA(c, cudaMalloc(&m, cap));
      c->weight_chunks.push_back(m);
      c->chunk_used = 0;
      c->chunk_cap = cap;
    }
    *p = reinterpret_cast<T*>(static_cast<char*>(c->weight_chunks.back()) + c->chunk_used);
    c->chunk_used += bytes;
    return VA_OK;
  }

  int find(const std::string& name, bool required, va::GgufTensorRef* t, bool* present) {
    const int rc = va::gguf_tensor_ref(g, name.c_str(), t);
    *present = rc == VA_OK;
    if (rc == VA_ERR_NOT_FOUND && !required) return VA_OK;
    return rc ? fail(c, rc, va::gguf_message()) : VA_OK;
  }

  // F32 values of the Weights entry (n of them); NULL when absent and optional.
  int vec(const std::string& name, int64_t n, bool required, float** dst) {
    *dst = nullptr;
    va::GgufTensorRef t;
    bool present;
    int rc = find(name, required, &t, &present);
    if (rc || !present) return rc;
    if (t.numel != n)
      return fail(c, VA_ERR_INVALID, name + ": " + std::to_string(t.numel) + " values, expected " + std::to_string(n));
    int rc2;
    if ((rc2 = carve(dst, static_cast<size_t>(n)))) return rc2;
    if (t.ndims == 2)
      VA_CUDA(c, st.convert(t, t.shape[0], t.shape[1], t.shape[0], true, false, *dst));
    else
      VA_CUDA(c, st.convert(t, 1, n, n, false, false, *dst));
    return VA_OK;
  }

  // Linear weight in -> out features as the bf16 K-major operand [out][in]: a
  // rank-2 tensor's stored [out, in] is that operand; flat content is [in, out].
  int linear(const std::string& name, int64_t in, int64_t out, __nv_bfloat16** dst) {
    va::GgufTensorRef t;
    bool present;
    int rc = find(name, true, &t, &present);
    if (rc) return rc;
    if (t.numel != in * out || (t.ndims == 2 && (t.shape[0] != out || t.shape[1] != in)))
      return fail(c, VA_ERR_INVALID, name + ": shape does not match [" + std::to_string(out) + ", " +
                                         std::to_string(in) + "]");
    if ((rc = carve(dst, static_cast<size_t>(in * out)))) return rc;
    if (t.ndims == 2)
      VA_CUDA(c, st.convert(t, out, in, in, false, true, *dst));
    else
      VA_CUDA(c, st.convert(t, in, out, in, true, true, *dst));
    return VA_OK;
  }

  int layer(int i) {
    const int E = c->cfg.embed_dim, hd = c->cfg.head_dim;
    const std::string p = "vit.blk." + std::to_string(i) + ".";
    LayerWeights& l = c->layers[i];
    free_layer(l);
    l.in_arena = true;
    int rc;
    if ((rc = linear(p + "attn_qkv.weight", E, 3 * E, &l.w_qkv_t))) return rc;
    if ((rc = vec(p + "attn_qkv.bias", 3 * E, true, &l.qkv_b))) return rc;
    if ((rc = linear(p + "attn_proj.weight", E, E, &l.w_proj_t))) return rc;
    if ((rc = vec(p + "attn_proj.bias", E, true, &l.proj_b))) return rc;
    if ((rc = vec(p + "ls1", E, false, &l.ls1))) return rc;
    if ((rc = vec(p + "norm1.weight", E, false, &l.norm1_w))) return rc;
    if ((rc = vec(p + "norm1.bias", E, false, &l.norm1_b))) return rc;
    if ((rc = vec(p + "attn_qnorm.weight", hd, false, &l.qn_g))) return rc;
    if ((rc = vec(p + "attn_qnorm.bias", hd, false, &l.qn_b))) return rc;
    if ((rc = vec(p + "attn_knorm.weight", hd, false, &l.kn_g))) return rc;
    if ((rc = vec(p + "attn_knorm.bias", hd, false, &l.kn_b))) return rc;
    if ((l.qn_g == nullptr) != (l.kn_g == nullptr) || (l.qn_g && (!l.qn_b || !l.kn_b)))
      return fail(c, VA_ERR_INVALID, p + "attn_qnorm/attn_knorm tensors must be given together");
    if ((l.norm1_w == nullptr) != (l.norm1_b == nullptr))
      return fail(c, VA_ERR_INVALID, p + "norm1 weight and bias must be given together");
    l.loaded = true;
    return VA_OK;
  }

  int mlp(int i, const va::GgufTensorRef& fc1) {
    const int E = c->cfg.embed_dim;
    const std::string p = "vit.blk." + std::to_string(i) + ".";
    const int64_t hidden = fc1.numel / E;
    if (fc1.numel % E != 0 || hidden <= 0 || hidden % 256 != 0 || hidden > (1 << 20))
      return fail(c, VA_ERR_INVALID, p + "mlp_fc1.weight: hidden width must be a positive multiple of 256");
    MlpWeights& m = c->mlps[i];
    free_mlp(m);
    m.in_arena = true;
    if (hidden > c->hidden_cap) {
      dfree(c->hbuf);
      VA_CUDA(c, dmalloc(&c->hbuf, static_cast<size_t>(c->cap) * hidden));
      c->hidden_cap = static_cast<int>(hidden);
    }
    int rc;
    if ((rc = vec(p + "norm2.weight", E, true, &m.norm2_w))) return rc;
    if ((rc = vec(p + "norm2.bias", E, true, &m.norm2_b))) return rc;
    if ((rc = linear(p + "mlp_fc1.weight", E, hidden, &m.w_fc1_t))) return rc;
    if ((rc = vec(p + "mlp_fc1.bias", hidden, true, &m.fc1_b))) return rc;
    if ((rc = linear(p + "mlp_fc2.weight", hidden, E, &m.w_fc2_t))) return rc;
    if ((rc = vec(p + "mlp_fc2.bias", E, true, &m.fc2_b))) return rc;
    if ((rc = vec(p + "ls2", E, false, &m.ls2))) return rc;
    m.hidden = static_cast<int>(hidden);
    m.loaded = true;
    return VA_OK;
  }

  // va_load_patch_embed's set (patch_embed.rs:150-198, pos_embed.rs:89-106).
  int patch_embed(const va::GgufTensorRef& w) {
    const int E = c->cfg.embed_dim;
    const int64_t features = w.numel / E;
    const int patch = static_cast<int>(std::lround(std::sqrt(static_cast<double>(features) / 3.0)));
    if (w.numel % E != 0 || patch <= 0 || 3LL * patch * patch != features || features > 4096 ||
        (w.ndims == 4 && (w.shape[0] != E || w.shape[1] != 3 || w.shape[2] != patch || w.shape[3] != patch)) ||
        (w.ndims == 2 && w.shape[1] != E))
      return fail(c, VA_ERR_INVALID, "vit.patch_embed.weight: shape is not [embed_dim, 3, p, p]");
    free_patch_embed(c);
    PatchEmbedWeights& p = c->pe;
    p.in_arena = true;
    const int kp = static_cast<int>((features + 63) / 64 * 64);
    int rc;
    if ((rc = carve(&p.w_t, static_cast<size_t>(E) * kp))) return rc;
    if (kp > features) VA_CUDA(c, st.zero(p.w_t, static_cast<size_t>(E) * kp * sizeof(__nv_bfloat16)));
    // OIHW content [E][3*p*p] is the K-major operand, padded to kp columns.
    if (w.ndims == 2)
      VA_CUDA(c, st.convert(w, w.shape[0], w.shape[1], kp, true, true, p.w_t));
    else
      VA_CUDA(c, st.convert(w, E, features, kp, false, true, p.w_t));
    if ((rc = vec("vit.patch_embed.bias", E, true, &p.bias))) return rc;
    if ((rc = vec("vit.cls_token", E, true, &p.cls))) return rc;
    va::GgufTensorRef pos;
    bool present;
    if ((rc = find("vit.pos_embed", true, &pos, &present))) return rc;
    const int64_t pos_rows = pos.numel / E;
    const int grid = static_cast<int>(std::llround(std::sqrt(static_cast<double>(std::max<int64_t>(pos_rows - 1, 0)))));
    if (pos.numel % E != 0 || pos_rows < 2 || static_cast<int64_t>(grid) * grid != pos_rows - 1)
      return fail(c, VA_ERR_INVALID, "vit.pos_embed: patch-row count is not a perfect square");
    if ((rc = vec("vit.pos_embed", pos.numel, true, &p.pos))) return rc;
    const int nr = c->cfg.num_register;
    if (nr > 0 && (rc = vec("vit.register_tokens", static_cast<int64_t>(nr) * E, true, &p.regs))) return rc;
    if (kp > E) VA_CUDA(c, dmalloc(&p.rows, static_cast<size_t>(c->cap) * kp));
    p.patch = patch;
    p.kp = kp;
    p.grid = grid;
    p.n_register = nr;
    p.offset = 0.1f;
    p.loaded = true;
    return VA_OK;
  }
};

}  // namespace

extern "C" {

int va_load_model_gguf(va_ctx* c, const va_gguf* g, int64_t* uploaded_bytes) {
  if (!c) return VA_ERR_INVALID;
  if (!g) return fail(c, VA_ERR_INVALID, "null model file");
  VA_CUDA(c, cudaSetDevice(c->device));
  VA_CUDA(c, cudaDeviceSynchronize());  // earlier calls may still read the weights being replaced
  // A model file replaces everything the previous one loaded: release the sets that
  // still point into the old arena, then the arena itself.
  for (auto& l : c->layers)
    if (l.in_arena) free_layer(l);
  for (auto& m : c->mlps)
    if (m.in_arena) free_mlp(m);
  if (c->pe.in_arena) free_patch_embed(c);
  if (c->vit_norm_in_arena) free_vit_norm(c);
  for (void* chunk : c->weight_chunks) cudaFree(chunk);
  c->weight_chunks.clear();
  c->chunk_used = c->chunk_cap = 0;
  GgufLoad L{c, g, {}};
  int rc;
  va::GgufTensorRef t;
  for (int i = 0; i < c->cfg.depth; ++i) {
    const std::string p = "vit.blk." + std::to_string(i) + ".";
    if (va::gguf_tensor_ref(g, (p + "attn_qkv.weight").c_str(), &t) == VA_ERR_NOT_FOUND) continue;
    if ((rc = L.layer(i))) return rc;
    rc = va::gguf_tensor_ref(g, (p + "mlp_fc1.weight").c_str(), &t);
    if (rc == VA_ERR_NOT_FOUND) continue;
    if (rc) return fail(c, rc, va::gguf_message());
    if ((rc = L.mlp(i, t))) return rc;
  }
  rc = va::gguf_tensor_ref(g, "vit.patch_embed.weight", &t);
  if (rc != VA_ERR_NOT_FOUND) {
    if (rc) return fail(c, rc, va::gguf_message());
    if ((rc = L.patch_embed(t))) return rc;
  }
  if (va::gguf_tensor_ref(g, "vit.norm.weight", &t) != VA_ERR_NOT_FOUND) {
    free_vit_norm(c);
    c->vit_norm_in_arena = true;
    if ((rc = L.vec("vit.norm.weight", c->cfg.embed_dim, true, &c->vit_norm_w))) return rc;
    if ((rc = L.vec("vit.norm.bias", c->cfg.embed_dim, true, &c->vit_norm_b))) return rc;
  }
  VA_CUDA(c, L.st.finish());
  for (auto& l : c->layers) {
    if (!l.in_arena || !l.qn_g) continue;
    float h[4][64];
    const float* src[4] = {l.qn_g, l.qn_b, l.kn_g, l.kn_b};
    for (int i = 0; i < 4; ++i) VA_CUDA(c, cudaMemcpy(h[i], src[i], sizeof(h[i]), cudaMemcpyDeviceToHost));
    l.qk_bound = qk_bound_log2(h[0], h[1], h[2], h[3], 64);
  }
  if (uploaded_bytes) *uploaded_bytes = static_cast<int64_t>(L.st.uploaded);
  return VA_OK;
}

int va_pos_embed_device(va_ctx* c, int gh, int gw, float* out, void* stream) {
  if (!c || !out) return VA_ERR_INVALID;
  if (!c->pe.loaded) return fail(c, VA_ERR_STATE, "patch embedding not loaded (va_load_patch_embed)");
  if (gh <= 0 || gw <= 0) return fail(c, VA_ERR_INVALID, "empty patch grid");
  VA_CUDA(c, cudaSetDevice(c->device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float* table = nullptr;
  int rc = ensure_pos_table(c, gh, gw, st, &table);
  if (rc) return rc;
  VA_CUDA(c, cudaMemcpyAsync(out, table, static_cast<size_t>(1 + gh * gw) * c->cfg.embed_dim * sizeof(float),
                             cudaMemcpyDeviceToDevice, st));
  return VA_OK;
}

int va_prepare_tokens_device(va_ctx* c, const float* image, int views, int height, int width,
                             const float* position, float* tokens, void* stream) {
  if (!c || !image || !tokens) return VA_ERR_INVALID;
  const PatchEmbedWeights& p = c->pe;
  if (!p.loaded) return fail(c, VA_ERR_STATE, "patch embedding not loaded (va_load_patch_embed)");
  if (views <= 0 || height <= 0 || width <= 0 || height % p.patch || width % p.patch)
    return fail(c, VA_ERR_INVALID, "height and width must be positive multiples of patch_size");
  const int gh = height / p.patch, gw = width / p.patch;
  const int64_t n_patches = static_cast<int64_t>(gh) * gw;
  if (static_cast<int64_t>(views) * n_patches > c->cap)
    return fail(c, VA_ERR_INVALID, "views * patches exceed the context's max_rows");
  if ((reinterpret_cast<uintptr_t>(tokens) | reinterpret_cast<uintptr_t>(position)) & 15)
    return fail(c, VA_ERR_INVALID, "tokens and position must be 16-byte aligned");
  VA_CUDA(c, cudaSetDevice(c->device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float* pos = position;
  int rc;
  if (!pos && (rc = ensure_pos_table(c, gh, gw, st, &pos))) return rc;
  const int E = c->cfg.embed_dim, n_special = 1 + p.n_register;
  const int n_tok = n_special + static_cast<int>(n_patches);
  __nv_bfloat16* rows = p.rows ? p.rows : c->x;
  const bool band = va::patchify_band_fits(width, p.patch, p.kp) && (reinterpret_cast<uintptr_t>(image) & 15) == 0;
  if (band)
    VA_CUDA(c, va::launch_patchify_band(image, views, height, width, p.patch, p.kp, rows, p.cls, pos, p.regs,
                                        p.n_register, n_tok, E, tokens, st));
  else
    VA_CUDA(c, va::launch_patchify(image, views, height, width, p.patch, p.kp, rows, st));
  va::PatchEpilogueArgs ea{};
  ea.bias = p.bias;
  ea.pos = pos;
  ea.out = tokens;
  ea.rows = static_cast<int>(views * n_patches);
  ea.n_patches = static_cast<int>(n_patches);
  ea.n_tok = n_tok;
  ea.n_special = n_special;
  ea.embed = E;
  VA_CUDA(c, va::launch_patch_gemm(rows, p.w_t, p.kp, ea, c->err, st));
  if (!band)
    VA_CUDA(c, va::launch_token_specials(p.cls, pos, p.regs, p.n_register, views, n_tok, E, tokens, st));
  return VA_OK;
}

int va_prepare_tokens_host(va_ctx* c, const float* image, int views, int height, int width,
                           const float* position, float* tokens) {
  if (!c || !image || !tokens) return VA_ERR_INVALID;
  const PatchEmbedWeights& p = c->pe;
  if (!p.loaded) return fail(c, VA_ERR_STATE, "patch embedding not loaded (va_load_patch_embed)");
  if (views <= 0 || height <= 0 || width <= 0 || height % p.patch || width % p.patch)
    return fail(c, VA_ERR_INVALID, "height and width must be positive multiples of patch_size");
  const int E = c->cfg.embed_dim;
  const int64_t n_patches = static_cast<int64_t>(height / p.patch) * (width / p.patch);
  const int64_t n_tok = 1 + p.n_register + n_patches;
  const size_t img_elems = static_cast<size_t>(views) * 3 * height * width;
  const size_t tok_elems = static_cast<size_t>(views) * n_tok * E;
  const size_t staging = static_cast<size_t>(c->cap) * E;
  if (img_elems > staging || tok_elems > staging)
    return fail(c, VA_ERR_INVALID, "image or tokens exceed the host staging buffers (max_rows * E floats)");
  VA_CUDA(c, cudaSetDevice(c->device));
  float* pos_dev = nullptr;
  const size_t pos_elems = static_cast<size_t>(1 + n_patches) * E;
  if (position) {
    VA_CUDA(c, dmalloc(&pos_dev, pos_elems));
    VA_CUDA(c, cudaMemcpy(pos_dev, position, pos_elems * sizeof(float), cudaMemcpyHostToDevice));
  }
  int rc = VA_OK;
  cudaError_t e = cudaMemcpyAsync(c->in_f32, image, img_elems * sizeof(float), cudaMemcpyHostToDevice, c->stream);
  if (e != cudaSuccess) rc = cuda_fail(c, e, "image upload");
  if (!rc) rc = va_prepare_tokens_device(c, c->in_f32, views, height, width, pos_dev, c->out_f32, c->stream);
  if (!rc) {
    e = cudaMemcpyAsync(tokens, c->out_f32, tok_elems * sizeof(float), cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) rc = cuda_fail(c, e, "token download");
  }
  if (pos_dev) {
    cudaStreamSynchronize(c->stream);
    dfree(pos_dev);
  }
  if (rc) return rc;
  return read_device_error(c);
}

int va_backbone_device(va_ctx* c, float* tokens_dev, int64_t rows, int gh, int gw, int view_count,
                       int first_layer, int last_layer, int alt_start, int cat_token,
                       const float* camera_dev, int n_out, const int* out_layers,
                       float* const* feat_dev, float* const* cam_dev, void* stream) {
  return va_backbone_device_sharded(c, tokens_dev, rows, 0, rows, gh, gw, view_count, first_layer,
                                    last_layer, alt_start, cat_token, camera_dev, n_out, out_layers,
                                    feat_dev, cam_dev, stream);
}

int va_backbone_device_sharded(va_ctx* c, float* tokens_local, int64_t local_rows,
                               int64_t row_offset, int64_t window_rows, int gh, int gw,
                               int view_count, int first_layer, int last_layer, int alt_start,
                               int cat_token, const float* camera_dev, int n_out,
                               const int* out_layers, float* const* feat_dev,
                               float* const* cam_dev, void* stream) {
  if (!c || !tokens_local || view_count <= 0) return VA_ERR_INVALID;
  if (first_layer < 0 || last_layer > c->cfg.depth || first_layer >= last_layer)
    return fail(c, VA_ERR_INVALID, "layer range out of bounds");
  if (n_out < 0 || (n_out > 0 && (!out_layers || !feat_dev || !cam_dev)))
    return fail(c, VA_ERR_INVALID, "captures need out_layers, feat and cam buffers");
  if (n_out > 0 && !c->vit_norm_w) return fail(c, VA_ERR_STATE, "captures need va_load_vit_norm");
  const int n_special = 1 + c->cfg.num_register;
  const int64_t n = n_special + static_cast<int64_t>(gh) * gw;
  if (n * view_count != window_rows) return fail(c, VA_ERR_INVALID, "window_rows must equal view_count * tokens per view");
  if (local_rows <= 0 || local_rows % n || row_offset % n || row_offset < 0 ||
      row_offset + local_rows > window_rows)
    return fail(c, VA_ERR_INVALID, "a rank's slice must hold whole views of the window");
  const bool sharded = local_rows != window_rows;
  for (int i = 0; i < n_out; ++i)
    if (!feat_dev[i] || !cam_dev[i]) return fail(c, VA_ERR_INVALID, "missing capture buffer");
  auto is_global = [&](int l) { return alt_start >= 0 && l >= alt_start && l % 2 == 1; };
  if (sharded) {
    bool any_global = false;
    for (int l = first_layer; l < last_layer; ++l) any_global |= is_global(l);
    if (any_global && !c->comm) return fail(c, VA_ERR_STATE, "global blocks over a sharded window need va_comm_init");
    // The NCCL fallback needs equal slices; view-aligned uneven slices need the
    // direct exchange.
    if (any_global && !c->p2p && window_rows != local_rows * va::comm_size(c->comm))
      return fail(c, VA_ERR_STATE, "uneven view slices need the direct K'/V exchange");
  }
  VA_CUDA(c, cudaSetDevice(c->device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int E = c->cfg.embed_dim;
  const int local_views = static_cast<int>(local_rows / n);
  bool snap_valid = false;
  for (int layer = first_layer; layer < last_layer; ++layer) {
    const bool global = is_global(layer);
    if (camera_dev && layer == alt_start)
      VA_CUDA(c, va::launch_camera_inject(tokens_local, camera_dev, local_views, static_cast<int>(n), E, st,
                                          row_offset == 0));
    if (layer < 0 || !c->mlps[layer].loaded) return fail(c, VA_ERR_STATE, "MLP weights not loaded (va_load_mlp)");
    int rc;
    if (global && sharded) {
      // Query-sharded global block over the whole window, then the token-local MLP.
      rc = device_call(c, layer, tokens_local, true, tokens_local, tokens_local, window_rows, local_rows,
                       row_offset, gh, gw, view_count, 1, true, st);
      if (!rc) rc = run_mlp(c, layer, tokens_local, local_rows, st);
    } else {
      // Local blocks (and every block on one GPU) run on the rank's own views.
      rc = va_block_device(c, layer, tokens_local, local_rows, gh, gw, global ? view_count : local_views,
                           global ? 1 : 0, st);
    }
    if (rc) return rc;
    for (int i = 0; i < n_out; ++i) {
      if (out_layers[i] != layer) continue;
      if (global && cat_token && !snap_valid)
        return fail(c, VA_ERR_STATE, "a global capture needs the preceding local block in the range");
      const float* local = global ? c->local_snap : tokens_local;
      VA_CUDA(c, va::launch_capture(tokens_local, local, c->vit_norm_w, c->vit_norm_b, c->cfg.ln_eps,
                                    local_views, static_cast<int>(n), n_special, E, cat_token ? 1 : 0,
                                    feat_dev[i], cam_dev[i], st));
    }
    if (!global && layer + 1 < last_layer && is_global(layer + 1)) {
      if (!c->local_snap) VA_CUDA(c, dmalloc(&c->local_snap, static_cast<size_t>(c->cap) * E));
      VA_CUDA(c, cudaMemcpyAsync(c->local_snap, tokens_local, static_cast<size_t>(local_rows) * E * sizeof(float),
                                 cudaMemcpyDeviceToDevice, st));
      snap_valid = true;
    }
  }
  return VA_OK;
}

int va_block_device_sharded(va_ctx* c, int layer, float* tokens_local, int64_t local_rows, int gh,
                            int gw, int view_count, int global, void* stream) {
  if (!c || !tokens_local) return VA_ERR_INVALID;
  if (layer < 0 || layer >= c->cfg.depth || !c->mlps[layer].loaded)
    return fail(c, VA_ERR_STATE, "MLP weights not loaded (va_load_mlp)");
  const int nranks = c->comm ? va::comm_size(c->comm) : 1;
  const int rank = c->comm ? va::comm_rank(c->comm) : 0;
  if (global && !c->comm) return fail(c, VA_ERR_STATE, "no communicator (va_comm_init)");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = device_call(c, layer, tokens_local, true, tokens_local, tokens_local, local_rows * nranks,
                       local_rows, local_rows * rank, gh, gw, view_count, global, true, st);
  if (rc) return rc;
  return run_mlp(c, layer, tokens_local, local_rows, st);
}

int va_run_tail_host(va_ctx* c, int layer, const float* tokens, int64_t rows, int gh, int gw,
                     int view_count, int global, float* out) {
  if (!c || !tokens || !out) return VA_ERR_INVALID;
  if (rows <= 0 || rows > c->cap) return fail(c, VA_ERR_INVALID, "rows out of range");
  VA_CUDA(c, cudaSetDevice(c->device));
  const size_t bytes = static_cast<size_t>(rows) * c->cfg.embed_dim * sizeof(float);
  VA_CUDA(c, cudaMemcpyAsync(c->in_f32, tokens, bytes, cudaMemcpyHostToDevice, c->stream));
  int rc = va_block_device(c, layer, c->in_f32, rows, gh, gw, view_count, global, c->stream);
  if (rc) {
    cudaStreamSynchronize(c->stream);
    return rc;
  }
  VA_CUDA(c, cudaMemcpyAsync(out, c->in_f32, bytes, cudaMemcpyDeviceToHost, c->stream));
  VA_CUDA(c, cudaStreamSynchronize(c->stream));
  return read_device_error(c);
}

int va_comm_unique_id(void* id_out) {
  if (!id_out) return VA_ERR_INVALID;
  std::string err;
  return va::comm_unique_id(id_out, &err) ? VA_OK : VA_ERR_NCCL;
}

int va_comm_init(va_ctx* c, const void* id, int nranks, int rank) {
  if (!c || !id || nranks <= 0 || rank < 0 || rank >= nranks) return VA_ERR_INVALID;
  VA_CUDA(c, cudaSetDevice(c->device));
  if (c->comm) {
    close_peers(c);
    va::comm_destroy(c->comm, false);
    c->comm = nullptr;
  }
  std::string err;
  c->comm = va::comm_init(id, nranks, rank, &err);
  if (!c->comm) return fail(c, VA_ERR_NCCL, err);
  return setup_peers(c);
}

int va_comm_exchange_mode(const va_ctx* c) {
  if (!c || !c->comm) return 0;
  return c->ce ? 3 : c->p2p ? 2 : 1;
}

int va_attention_device_sharded(va_ctx* c, int layer, const float* ln1_local, float* out_local,
                                int64_t local_rows, int gh, int gw, int view_count, int global,
                                void* stream) {
  if (!c || !ln1_local || !out_local) return VA_ERR_INVALID;
  const int nranks = c->comm ? va::comm_size(c->comm) : 1;
  const int rank = c->comm ? va::comm_rank(c->comm) : 0;
  if (global && !c->comm) return fail(c, VA_ERR_STATE, "no communicator (va_comm_init)");
  return device_call(c, layer, ln1_local, false, out_local, nullptr, local_rows * nranks, local_rows,
                     local_rows * rank, gh, gw, view_count, global, true,
                     static_cast<cudaStream_t>(stream));
}

int va_op_attention_device(va_ctx* c, const float* q, const float* k, const float* v, int heads,
                           int64_t n, int head_dim, const float* qn_g, const float* qn_b,
                           const float* kn_g, const float* kn_b, float qk_norm_eps,
                           const float* pos_yx_host, float freq, float* out, void* stream) {
  if (!c || !q || !k || !v || !out) return VA_ERR_INVALID;
  if (head_dim != 64) return fail(c, VA_ERR_INVALID, "Op::Attention on device needs head_dim 64");
  if (heads <= 0 || n <= 0 || static_cast<int64_t>(heads) * n > 0x7fffffff / 64)
    return fail(c, VA_ERR_INVALID, "bad heads/n");
  if ((qn_g == nullptr) != (qn_b == nullptr) || (kn_g == nullptr) != (kn_b == nullptr))
    return fail(c, VA_ERR_INVALID, "norm gamma and beta must be given together");
  if (pos_yx_host && freq != c->cfg.rope_freq)
    return fail(c, VA_ERR_INVALID, "RoPE base must equal the context's rope_freq");
  VA_CUDA(c, cudaSetDevice(c->device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t per = static_cast<size_t>(heads) * n * 64;
  if (3 * per > c->op_cap) {
    dfree(c->op_buf);
    VA_CUDA(c, dmalloc(&c->op_buf, 3 * per));
    c->op_cap = 3 * per;
  }
  int2* pos = nullptr;
  if (pos_yx_host) {
    if (static_cast<size_t>(n) > c->op_pos_cap) {
      dfree(c->op_pos);
      VA_CUDA(c, dmalloc(&c->op_pos, static_cast<size_t>(n)));
      c->op_pos_cap = n;
    }
    VA_CUDA(c, cudaStreamSynchronize(st));  // op_pos may still be read by an earlier call
    int rc = upload_positions(c, pos_yx_host, n, c->op_pos);
    if (rc) return rc;
    pos = c->op_pos;
  }
  __nv_bfloat16* qb = c->op_buf;
  __nv_bfloat16* kb = c->op_buf + per;
  __nv_bfloat16* vb = c->op_buf + 2 * per;
  VA_CUDA(c, va::launch_prep_heads(q, heads, static_cast<int>(n), qn_g, qn_b, qk_norm_eps, pos,
                                   c->rope_cs, c->cfg.rope_pairing, qb, st));
  VA_CUDA(c, va::launch_prep_heads(k, heads, static_cast<int>(n), kn_g, kn_b, qk_norm_eps, pos,
                                   c->rope_cs, c->cfg.rope_pairing, kb, st));
  VA_CUDA(c, va::launch_prep_heads(v, heads, static_cast<int>(n), nullptr, nullptr, 0.f, nullptr,
                                   nullptr, 0, vb, st));
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
  fa.v_f16 = 0;
  set_split_workspace(c, &fa);
  VA_CUDA(c, va::launch_flash(qb, kb, vb, fa, c->err, st));
  return VA_OK;
}

int va_flash_attention_bf16(va_ctx* c, const void* q, const void* k, const void* v,
                            int64_t q_count, int64_t q_offset, int64_t kv_rows, int heads,
                            int64_t seg_len, int v_f16, int variant, void* out,
                            void* stream) {
  if (!c || !q || !k || !v || !out) return VA_ERR_INVALID;
  if (q_count <= 0 || kv_rows <= 0 || heads <= 0 || seg_len < 0 || q_offset < 0 ||
      kv_rows > 0x7fffffff / 64 / heads || q_count > kv_rows)
    return fail(c, VA_ERR_INVALID, "bad flash shape");
  if (seg_len > 0 && (q_count % seg_len || q_offset % seg_len || q_offset + q_count > kv_rows))
    return fail(c, VA_ERR_INVALID, "local attention needs whole segments inside the key rows");
  va::FlashArgs fa{};
  fa.q_count = static_cast<int>(q_count);
  fa.q_offset = static_cast<int>(q_offset);
  fa.kv_rows = static_cast<int>(kv_rows);
  fa.seg_len = static_cast<int>(seg_len);
  fa.heads = heads;
  fa.scale_log2 = static_cast<float>(1.0 / 8.0 * 1.4426950408889634);
  fa.out_mode = 0;
  fa.o_tok = static_cast<__nv_bfloat16*>(out);
  fa.embed = heads * 64;
  fa.v_f16 = v_f16 ? 1 : 0;
  if (variant >= 256) {  // caller guarantees |q.k| * scale * log2(e) <= 64
    if (v_f16) return fail(c, VA_ERR_INVALID, "the fixed exponent offset needs bf16 V");
    fa.fixed_offset = 1;
    variant -= 256;
    if (variant == 255) variant = -1;  // 511: fixed offset with the library's default layout
  }
  if (variant >= 0) {
    const int poly = variant & 7, form = variant >> 3;
    const bool key_split = form >= 9 && form <= 15 && poly <= (form == 15 ? 2 : 4) && fa.fixed_offset;
    if (!key_split && (poly > 2 || form > 8 || (form == 8 && poly != 0)))
      return fail(c, VA_ERR_INVALID,
                  "variant must be poly (0..2) + 8 * form (0..7), 64, or with the fixed offset 8 * (9..14) + (0..4) or 8 * 15 + (0..2)");
    fa.poly_per8 = variant;
  }
  set_split_workspace(c, &fa);
  VA_CUDA(c, va::launch_flash(static_cast<const __nv_bfloat16*>(q),
                              static_cast<const __nv_bfloat16*>(k),
                              static_cast<const __nv_bfloat16*>(v), fa, c->err,
                              static_cast<cudaStream_t>(stream)));
  return VA_OK;
}

int va_flash_plan(int64_t q_count, int64_t q_offset, int64_t kv_rows, int heads, int64_t seg_len,
                  int fixed_offset, int variant, int sms, int* plan) {
  if (!plan || sms <= 0 || heads <= 0 || heads > 64 || q_count <= 0 || kv_rows <= 0 || q_offset < 0 ||
      seg_len < 0 || q_count > 0x7fffffff || kv_rows > 0x7fffffff || q_offset > 0x7fffffff ||
      seg_len > 0x7fffffff)
    return VA_ERR_INVALID;
  va::FlashArgs fa{};
  fa.q_count = static_cast<int>(q_count);
  fa.q_offset = static_cast<int>(q_offset);
  fa.kv_rows = static_cast<int>(kv_rows);
  fa.seg_len = static_cast<int>(seg_len);
  fa.heads = heads;
  fa.embed = heads * 64;
  fa.fixed_offset = fixed_offset ? 1 : 0;
  if (variant >= 256) {  // as va_flash_attention_bf16: + 256 = the fixed exponent offset
    fa.fixed_offset = 1;
    variant -= 256;
    if (variant == 255) variant = -1;
  }
  fa.poly_per8 = variant < 0 ? -1 : variant;
  fa.sms = sms;
  fa.part_slots = va::flash_part_slots(sms);
  va::FlashPlan p;
  if (va::flash_plan(fa, sms, 2, true, &p) != cudaSuccess) return VA_ERR_INVALID;
  const int v[9] = {p.form, p.poly, p.unit_rows, p.per_sm, fa.n_full, fa.splits, p.grid_x, p.grid_y, p.grid_z};
  for (int i = 0; i < 9; ++i) plan[i] = v[i];
  return VA_OK;
}

int va_linear_bf16(va_ctx* c, const void* a, const void* w_t, const float* bias, const float* scale,
                   const float* residual, float* out, int64_t m, int n, int k, void* stream) {
  if (!c || !a || !w_t || !out) return VA_ERR_INVALID;
  if (m <= 0 || m > 0x7fffffff || n % 128 != 0 || k % 64 != 0 || n <= 0 || k <= 0)
    return fail(c, VA_ERR_INVALID, "linear needs n % 128 == 0 and k % 64 == 0");
  va::ProjEpilogueArgs pa{};
  pa.bias = bias;
  pa.ls1 = scale;
  pa.residual = residual;
  pa.out = out;
  pa.rows = static_cast<int>(m);
  pa.embed = n;
  cudaError_t e = va::launch_proj_gemm(static_cast<const __nv_bfloat16*>(a),
                                       static_cast<const __nv_bfloat16*>(w_t), static_cast<int>(m),
                                       n, k, pa, c->err, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(c, e, "launch_proj_gemm");
  return VA_OK;
}

int va_select_reference_view_saddle(const float* cls, int views, int embed, int* out_index) {
  if (!cls || !out_index || views <= 0) return VA_ERR_INVALID;
  if (views == 1) {
    *out_index = 0;
    return VA_OK;
  }
  if (embed <= 1) return VA_ERR_INVALID;
  // backbone.rs:133-206: normalised CLS rows, mean cosine similarity to the other
  // views, vector norm and unbiased variance of the normalised row; each min-max
  // normalised (denominator + 1e-8); the view minimising the summed distance to
  // 0.5 wins, ties keep the earliest view.
  std::vector<double> norm(views), sim(views, 0.0), var(views, 0.0);
  std::vector<double> nz(static_cast<size_t>(views) * embed);
  for (int v = 0; v < views; ++v) {
    double s = 0.0;
    for (int e = 0; e < embed; ++e) {
      const double x = cls[static_cast<size_t>(v) * embed + e];
      s += x * x;
    }
    const double mag = std::sqrt(s);
    norm[v] = mag;
    const double inv = mag > 0.0 ? 1.0 / mag : 0.0;
    for (int e = 0; e < embed; ++e)
      nz[static_cast<size_t>(v) * embed + e] = static_cast<double>(cls[static_cast<size_t>(v) * embed + e]) * inv;
  }
  for (int v = 0; v < views; ++v) {
    for (int o = 0; o < views; ++o) {
      if (o == v) continue;
      double d = 0.0;
      for (int e = 0; e < embed; ++e) d += nz[static_cast<size_t>(v) * embed + e] * nz[static_cast<size_t>(o) * embed + e];
      sim[v] += d;
    }
    sim[v] /= static_cast<double>(views - 1);
    double mean = 0.0;
    for (int e = 0; e < embed; ++e) mean += nz[static_cast<size_t>(v) * embed + e];
    mean /= embed;
    double acc = 0.0;
    for (int e = 0; e < embed; ++e) {
      const double d = nz[static_cast<size_t>(v) * embed + e] - mean;
      acc += d * d;
    }
    var[v] = acc / static_cast<double>(embed - 1);
  }
  auto norm01 = [](std::vector<double>& x) {
    double lo = INFINITY, hi = -INFINITY;
    for (double y : x) {
      lo = std::min(lo, y);
      hi = std::max(hi, y);
    }
    const double den = hi - lo + 1e-8;
    for (double& y : x) y = (y - lo) / den;
  };
  norm01(sim);
  norm01(norm);
  norm01(var);
  int best = 0;
  double best_b = INFINITY;
  for (int v = 0; v < views; ++v) {
    const double b = std::fabs(sim[v] - 0.5) + std::fabs(norm[v] - 0.5) + std::fabs(var[v] - 0.5);
    if (b < best_b) {
      best_b = b;
      best = v;
    }
  }
  *out_index = best;
  return VA_OK;
}

int va_reference_first_order(int views, int reference, int* order_out) {
  if (!order_out || views <= 0 || reference < 0 || reference >= views) return VA_ERR_INVALID;
  int i = 0;
  order_out[i++] = reference;
  for (int v = 0; v < views; ++v)
    if (v != reference) order_out[i++] = v;
  return VA_OK;
}

int va_restore_order(int views, int reference, int* src_out) {
  if (!src_out || views <= 0 || reference < 0 || reference >= views) return VA_ERR_INVALID;
  // ordered position p holds original view order[p]; invert it.
  std::vector<int> order(views);
  va_reference_first_order(views, reference, order.data());
  for (int p = 0; p < views; ++p) src_out[order[p]] = p;
  return VA_OK;
}

int va_camera_inject_device(float* tokens_dev, const float* camera_dev, int views,
                            int64_t tokens_per_view, int embed, void* stream) {
  if (!tokens_dev || !camera_dev || views <= 0 || tokens_per_view <= 0 || embed <= 0 ||
      tokens_per_view > 0x7fffffff)
    return VA_ERR_INVALID;
  return va::launch_camera_inject(tokens_dev, camera_dev, views, static_cast<int>(tokens_per_view),
                                  embed, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? VA_OK
             : VA_ERR_CUDA;
}

int va_permute_views_device(const float* src_dev, float* dst_dev, const int* order_host, int views,
                            int64_t view_elems, void* stream) {
  if (!src_dev || !dst_dev || !order_host || views <= 0 || view_elems <= 0 || src_dev == dst_dev)
    return VA_ERR_INVALID;
  std::vector<int> seen(views, 0);
  for (int i = 0; i < views; ++i) {
    if (order_host[i] < 0 || order_host[i] >= views || seen[order_host[i]]++) return VA_ERR_INVALID;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* d_order = nullptr;
  if (cudaMallocAsync(reinterpret_cast<void**>(&d_order), sizeof(int) * views, st) != cudaSuccess)
    return VA_ERR_CUDA;
  if (cudaMemcpyAsync(d_order, order_host, sizeof(int) * views, cudaMemcpyHostToDevice, st) !=
      cudaSuccess)
    return VA_ERR_CUDA;
  const cudaError_t e = va::launch_permute_views(src_dev, dst_dev, d_order, views, view_elems, st);
  cudaFreeAsync(d_order, st);
  if (e != cudaSuccess) return VA_ERR_CUDA;
  // order_host is pageable: the H2D copy above completed before returning.
  return VA_OK;
}

int va_check_device(va_ctx* c) {
  if (!c) return VA_ERR_INVALID;
  VA_CUDA(c, cudaSetDevice(c->device));
  VA_CUDA(c, cudaDeviceSynchronize());
  return read_device_error(c);
}

int va_set_phase_profile(va_ctx* c, int enable) {
  if (!c) return VA_ERR_INVALID;
  c->phase_profile = enable != 0;
  c->phase_valid = false;
  return VA_OK;
}

int va_phase_times(va_ctx* c, float* ms_out) {
  if (!c || !ms_out) return VA_ERR_INVALID;
  if (!c->phase_valid) return fail(c, VA_ERR_STATE, "no profiled device-path call since the profile was enabled");
  VA_CUDA(c, cudaSetDevice(c->device));
  VA_CUDA(c, cudaEventSynchronize(c->ph_ev[kPhases]));
  for (int i = 0; i < kPhases; ++i) VA_CUDA(c, cudaEventElapsedTime(&ms_out[i], c->ph_ev[i], c->ph_ev[i + 1]));
  return VA_OK;
}

int va_last_exchange(const va_ctx* c) { return c ? c->last_xchg : 0; }

int va_exchange_times(va_ctx* c, float* ms_out, int* npeer_out, int64_t* bytes_per_peer) {
  if (!c || !ms_out || !npeer_out || !bytes_per_peer) return VA_ERR_INVALID;
  if (!c->phase_valid) return fail(c, VA_ERR_STATE, "no profiled device-path call since the profile was enabled");
  *npeer_out = 0;
  *bytes_per_peer = 0;
  if (c->xchg_peers == 0) return VA_OK;  // the last call pushed nothing by copy engines
  VA_CUDA(c, cudaSetDevice(c->device));
  for (int p = 0; p < c->xchg_peers; ++p) {
    VA_CUDA(c, cudaEventSynchronize(c->ce_t1[p]));
    VA_CUDA(c, cudaEventElapsedTime(&ms_out[p], c->ce_t0[p], c->ce_t1[p]));
  }
  *npeer_out = c->xchg_peers;
  *bytes_per_peer = c->xchg_bytes;
  return VA_OK;
}

int va_selftest_bounded_wait(va_ctx* c, int64_t limit_us) {
  if (!c) return VA_ERR_INVALID;
  if (limit_us <= 0 || limit_us > 1000000) return fail(c, VA_ERR_INVALID, "limit_us must be in (0, 1e6]");
  VA_CUDA(c, cudaSetDevice(c->device));
  VA_CUDA(c, cudaStreamSynchronize(c->stream));
  int rc = read_device_error(c);  // start from a clear error word
  if (rc) return rc;
  VA_CUDA(c, va::launch_bounded_wait_selftest(static_cast<unsigned long long>(limit_us) * 1000ull,
                                              c->err, c->stream));
  VA_CUDA(c, cudaStreamSynchronize(c->stream));
  return read_device_error(c);
}

int va_selftest_peer_wait(va_ctx* c, int peer_flag, float* out_max_abs) {
  if (!c) return VA_ERR_INVALID;
  VA_CUDA(c, cudaSetDevice(c->device));
  VA_CUDA(c, cudaStreamSynchronize(c->stream));
  int rc = read_device_error(c);
  if (rc) return rc;
  // One head, 256 keys of which this "rank 0 of 2" owns the first 128; rank 1's flag
  // is `peer_flag` against epoch 1.  Inputs are a fixed pattern; the result is
  // compared with the same launch without a peer.
  const int rows = 256, cols = 64;
  std::vector<uint16_t> h(static_cast<size_t>(rows) * cols);
  for (size_t i = 0; i < h.size(); ++i) h[i] = f32_to_bf16_rne(std::sin(0.37f * static_cast<float>(i)));
  __nv_bfloat16 *qkv = nullptr, *o1 = nullptr, *o2 = nullptr;
  unsigned long long* flags = nullptr;
  auto release = [&]() {
    cudaStreamSynchronize(c->stream);
    dfree(qkv);
    dfree(o1);
    dfree(o2);
    dfree(flags);
  };
  cudaError_t e = dmalloc(&qkv, h.size());
  if (e == cudaSuccess) e = dmalloc(&o1, h.size());
  if (e == cudaSuccess) e = dmalloc(&o2, h.size());
  if (e == cudaSuccess) e = dmalloc(&flags, va::kMaxRanks);
  if (e == cudaSuccess) e = cudaMemcpy(qkv, h.data(), h.size() * 2, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(flags, 0, va::kMaxRanks * sizeof(unsigned long long));
  const unsigned long long raised = va::peer_flag_value(1, true, rows);
  if (e == cudaSuccess && peer_flag) e = cudaMemcpy(flags + 1, &raised, sizeof(raised), cudaMemcpyHostToDevice);
  va::FlashArgs fa{};
  fa.q_count = rows;
  fa.kv_rows = rows;
  fa.heads = 1;
  fa.embed = cols;
  fa.scale_log2 = static_cast<float>(1.0 / 8.0 * 1.4426950408889634);
  fa.o_tok = o1;
  if (e == cudaSuccess) e = va::launch_flash(qkv, qkv, qkv, fa, c->err, c->stream);
  fa.o_tok = o2;
  fa.peer_flags = flags;
  fa.epoch = 1;
  fa.nranks = 2;
  fa.rank = 0;
  fa.own_begin = 0;
  fa.own_end = 128;
  if (e == cudaSuccess) e = va::launch_flash(qkv, qkv, qkv, fa, c->err, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) {
    release();
    return cuda_fail(c, e, "peer-wait self-test");
  }
  rc = read_device_error(c);
  if (rc == VA_OK && out_max_abs) {
    std::vector<uint16_t> a(h.size()), b(h.size());
    cudaMemcpy(a.data(), o1, a.size() * 2, cudaMemcpyDeviceToHost);
    cudaMemcpy(b.data(), o2, b.size() * 2, cudaMemcpyDeviceToHost);
    float m = 0.f;
    for (size_t i = 0; i < a.size(); ++i) {
      uint32_t ua = static_cast<uint32_t>(a[i]) << 16, ub = static_cast<uint32_t>(b[i]) << 16;
      float fa_, fb_;
      std::memcpy(&fa_, &ua, 4);
      std::memcpy(&fb_, &ub, 4);
      m = std::max(m, std::fabs(fa_ - fb_));
    }
    *out_max_abs = m;
  }
  release();
  return rc;
}

}  // extern "C"
