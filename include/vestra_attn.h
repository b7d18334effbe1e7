/*
 * vestra_attn.h -- C ABI of the B200 (sm_100a) attention path for the DA3 ViT
 * backbone of Vestra Engine.
 *
 * This library replaces, on the attention path, the opt-in CUDA oracle slice of
 * the reference (crates/da-engine/src/vit_block.rs:140-372, behind the
 * `cuda-residual-oracle` feature) and the CPU `vestra_kernels::attention`
 * call it falls back to.  A Rust FFI crate (vestra-cuda-sys) binds these symbols
 * one-to-one; see INTEGRATION.md for the binding and the executor adapter.
 *
 * Conventions
 *   - Every function returns an int status: VA_OK (0) or a VA_ERR_* code.  No
 *     exceptions or panics cross the boundary, and there is NO CPU fallback: an
 *     unsupported shape is VA_ERR_INVALID, never a silent host computation.
 *   - va_last_error(ctx) returns a message for the last failing call on ctx.
 *   - One context per host thread; calls on one context are serial (the
 *     reference's executors are called serially from the block loop).
 *   - Weight tensors use the reference's in-memory orientation: linear weights
 *     are [in, out] row-major F32 (engine.rs:110-126 transposes GGUF's [out, in]
 *     at load), vectors are F32.  The library converts and owns device copies.
 *   - `stream` arguments are cudaStream_t values passed as void*; NULL is the
 *     legacy default stream.
 *   - Tokens are view-major: view v occupies rows [v*n, (v+1)*n) with
 *     n = (1 + num_register) + gh*gw.
 */
#ifndef VESTRA_ATTN_H
#define VESTRA_ATTN_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VA_OK 0
#define VA_ERR_INVALID 1 /* unsupported shape / bad argument (reference executor: None) */
#define VA_ERR_CUDA 2    /* CUDA runtime failure */
#define VA_ERR_DEVICE 3  /* a kernel gave up on a bounded wait and set the error word */
#define VA_ERR_STATE 4   /* e.g. layer weights not loaded */
#define VA_ERR_NCCL 5    /* communicator failure */
#define VA_ERR_CAPACITY 6 /* request larger than a fixed-size buffer (va_op_attention_noalloc) */
#define VA_ERR_IO 7       /* GGUF: the file could not be opened or mapped (GgufError::Io) */
#define VA_ERR_FORMAT 8   /* GGUF: BadMagic, UnsupportedVersion or Malformed */
#define VA_ERR_NOT_FOUND 9 /* GGUF: TensorNotFound, or a metadata key absent / of another type */
#define VA_ERR_DTYPE 10   /* GGUF: UnsupportedDtype (tensor types other than F32, F16, Q8_0) */

typedef struct va_ctx va_ctx;

/* Fields read by the attention path from ModelConfig (config.rs:146, from_gguf
 * :219-264). */
typedef struct va_config {
  int32_t embed_dim;    /* E: 768 (DA3-BASE), 1024 (DA3-LARGE); multiple of 256 */
  int32_t num_heads;    /* H: embed_dim / 64 */
  int32_t head_dim;     /* must be 64 */
  int32_t depth;        /* number of blocks whose weights the context holds */
  int32_t num_register; /* special tokens per view = 1 + num_register (backbone.rs:347) */
  int32_t rope_start;   /* RoPE on blocks i >= rope_start; -1 = never (vit_block.rs:839) */
  int32_t qknorm_start; /* QK-norm on blocks i >= qknorm_start; -1 = never (:835-838) */
  float rope_freq;      /* RoPE base, 100 for DA3 (cfg.rope_freq) */
  float ln_eps;         /* block LayerNorm eps (cfg.ln_eps, 1e-6) */
  float qk_norm_eps;    /* per-head QK LayerNorm eps, 1e-5 (QK_NORM_EPS, vit_block.rs:686) */
  int32_t rope_pairing; /* 0: rotate-half pairs (i, i+16) per half (default); 1: interleaved */
  int32_t max_rows;     /* workspace capacity in tokens (rows per call) */
} va_config;

/* Library version string, e.g. "vestra_attn 0.1 sm_100a". */
const char* va_version(void);

/* DA3-BASE defaults: E=768, H=12, d=64, depth=12, num_register=0, rope/qknorm
 * start 4, rope_freq 100, ln_eps 1e-6, qk eps 1e-5, max_rows 12*866. */
void va_default_config(va_config* cfg);

/* Creates a context on CUDA device `device` and allocates its workspace.
 * Replaces CudaAttentionExecutor::new / CudaTransformerTailExecutor::new
 * (vit_block.rs:239-318, :375-397) together with the engine's
 * enable_cuda_attention_oracle(device) (engine.rs:323). */
int va_create(const va_config* cfg, int device, va_ctx** out);
void va_destroy(va_ctx* ctx);
const char* va_last_error(const va_ctx* ctx);

/* Uploads one block's attention weights (names from vit_block.rs:30-53):
 *   norm1_w/b [E]          vit.blk.{i}.norm1.{weight,bias}   (NULL: LN1 not fused)
 *   qkv_w [E,3E], qkv_b [3E]  vit.blk.{i}.attn_qkv.*  columns [Q|K|V], each [H,64]
 *   qnorm_w/b, knorm_w/b [64] vit.blk.{i}.attn_{q,k}norm.*    (NULL: absent tensor)
 *   proj_w [E,E], proj_b [E]  vit.blk.{i}.attn_proj.*
 *   ls1 [E]                vit.blk.{i}.ls1                   (NULL: absent tensor)
 * Mirrors the per-layer uploads of CudaAttentionExecutor::new (vit_block.rs:262-316). */
int va_load_layer(va_ctx* ctx, int layer, const float* norm1_w, const float* norm1_b,
                  const float* qkv_w, const float* qkv_b, const float* qnorm_w,
                  const float* qnorm_b, const float* knorm_w, const float* knorm_b,
                  const float* proj_w, const float* proj_b, const float* ls1);

/* Layer gating (vit_block.rs:835-839): use_qknorm = qknorm_start >= 0 && layer >=
 * qknorm_start && q-norm weights present; use_rope = rope_start >= 0 && layer >=
 * rope_start. */
int va_layer_flags(const va_ctx* ctx, int layer, int* use_qknorm, int* use_rope);

/* AttentionExecutor::run_attention (vit_block.rs:95-105, CUDA oracle :321-372):
 * input = LN1 output [rows, E] (host F32), positions_yx = [rows, 2] integer-valued
 * (y, x) as F32 or NULL (no RoPE), out = projected branch [rows, E] (host F32,
 * proj*ls1, no residual).  One attention over all rows (the caller's n).  QK-norm
 * follows the layer gating.  heads/head_dim must match the context. */
int va_run_attention(va_ctx* ctx, int layer, const float* input, int64_t rows, int heads,
                     int head_dim, const float* positions_yx, float* out);

/* run_attention with positions derived in closed form (vit_block.rs:841-881):
 * global = 1: one attention over all view_count*n rows, patch positions (1,1);
 * global = 0: view_count independent attentions (one per view), patch p at
 * (p/gw+1, p%gw+1).  Special tokens (0,0).  Host F32 in/out. */
int va_attention_host(va_ctx* ctx, int layer, const float* ln1, int64_t rows, int gh, int gw,
                      int view_count, int global, float* out);

/* va_attention_host over nsteps independent inputs of one shape (several requests'
 * windows, one layer), pipelined (no reference counterpart; the reference runs one
 * call at a time): step s+1's copy in runs beside step s's attention and copy out,
 * so both PCIe directions are busy at once, which a single call of a global block
 * cannot do (no output row is ready before its last input row has arrived).
 * ln1[s] / out[s]: host buffers [rows, E] (pinned for full speed); the results are
 * those of nsteps va_attention_host calls.  Single GPU; returns when all are done. */
int va_attention_host_batch(va_ctx* ctx, int layer, const float* const* ln1, float* const* out, int nsteps,
                            int64_t rows, int gh, int gw, int view_count, int global);

/* Same, device-resident: ln1_dev and out_dev are device F32 [rows, E]. */
int va_attention_device(va_ctx* ctx, int layer, const float* ln1_dev, float* out_dev,
                        int64_t rows, int gh, int gw, int view_count, int global, void* stream);

/* Attention half of vit_block_with_views (vit_block.rs:1058-1091) on device:
 * tokens += proj(attn(LN1(tokens))) * ls1, in place.  Needs norm1 weights. */
int va_block_attention_device(va_ctx* ctx, int layer, float* tokens_dev, int64_t rows, int gh,
                              int gw, int view_count, int global, void* stream);

/* Op::Attention (graph.rs:67-105; CpuBackend arm cpu_backend.rs:198-298) on device:
 * q, k, v, out [heads, n, 64] F32.  qn_g/qn_b/kn_g/kn_b [64] or NULL; pos_yx_host
 * [n, 2] host F32 (rounded) or NULL.  q and k are not modified. */
int va_op_attention_device(va_ctx* ctx, const float* q, const float* k, const float* v,
                           int heads, int64_t n, int head_dim, const float* qn_g,
                           const float* qn_b, const float* kn_g, const float* kn_b,
                           float qk_norm_eps, const float* pos_yx_host, float freq, float* out,
                           void* stream);

/* No counterpart in the reference: Op::Attention for callers that cannot allocate
 * device memory (a process whose allocator owns the whole GPU, or a block loop that
 * must not stall on cudaMalloc/cudaFree or fail on one).  Needs no context and
 * allocates nothing; its bf16 operand scratch is a fixed array of 12 MiB inside the
 * library, held on every GPU that loads it until exit.  All pointers are device
 * pointers: q, k, v, out [heads, n, 64] F32; norm vectors [64] or NULL; pos_yx_dev
 * [n, 2] F32 (rounded half away from zero; each in [0, 65535], else VA_ERR_INVALID) or
 * NULL; rope_pairing as in va_config.  Limit: heads * n * 64
 * <= 2,097,152, else VA_ERR_CAPACITY.  The first call on a device looks up the
 * scratch address with that device current.  Calls share the scratch: calls that
 * overlap on the GPU race.  The call waits for `stream` (it synchronizes it and reads
 * the device error word back) and returns VA_ERR_DEVICE if a kernel gave up on a
 * bounded wait. */
int va_op_attention_noalloc(const float* q, const float* k, const float* v, int heads,
                            int64_t n, int head_dim, const float* qn_g, const float* qn_b,
                            const float* kn_g, const float* kn_b, float qk_norm_eps,
                            const float* pos_yx_dev, float freq, int rope_pairing, float* out,
                            void* stream);

/* Transformer tail: the MLP sub-block and the whole block.
 * va_load_mlp replaces the CudaMlpExecutor weight upload (vit_block.rs:190-236):
 * norm2_w/b [E], fc1_w [E, mlp_hidden] and fc1_b [mlp_hidden], fc2_w [mlp_hidden, E]
 * and fc2_b [E] in the reference's [in, out] orientation, ls2 [E] or NULL
 * (presence-gated); mlp_hidden a multiple of 256 (4E for DA3).  The library copies
 * and converts the matrices to bf16. */
int va_load_mlp(va_ctx* ctx, int layer, int mlp_hidden, const float* norm2_w, const float* norm2_b,
                const float* fc1_w, const float* fc1_b, const float* fc2_w, const float* fc2_b,
                const float* ls2);
/* run_tail_device (vit_block.rs:489-583): one whole block in place on device tokens
 * F32 [rows, E]: x += proj(attention(LN1 x)) (*ls1); x += fc2(GELU_erf(fc1(LN2 x)))
 * (*ls2) (vit_block.rs:1019-1139).  Needs va_load_layer with norm1 and va_load_mlp. */
int va_block_device(va_ctx* ctx, int layer, float* tokens_dev, int64_t rows, int gh, int gw,
                    int view_count, int global, void* stream);
/* The same block over this rank's token slice of a query-sharded window (global
 * blocks exchange K'/V as va_attention_device_sharded does; the MLP is
 * token-local).  Collective for global blocks. */
int va_block_device_sharded(va_ctx* ctx, int layer, float* tokens_local, int64_t local_rows,
                            int gh, int gw, int view_count, int global, void* stream);
/* TransformerTailExecutor::run_tail (vit_block.rs:110-129) with host buffers:
 * tokens [rows, E] in, updated tokens out (may alias).  The reference's separate
 * CPU-order LN1 input is not taken: LN1 is computed on the device from tokens. */
int va_run_tail_host(va_ctx* ctx, int layer, const float* tokens, int64_t rows, int gh, int gw,
                     int view_count, int global, float* out);

/* Token input side: patch projection and CLS / register / position assembly on
 * the device, producing the view-major tokens va_backbone_device consumes.
 *
 * va_load_patch_embed replaces CudaPatchEmbedExecutor::new (patch_embed.rs:150-198)
 * and the weight lookups of prepare_tokens (pos_embed.rs:236-300): weight_oihw
 * vit.patch_embed.weight [E][3][patch][patch], bias vit.patch_embed.bias [E],
 * cls_token vit.cls_token [E], pos_embed vit.pos_embed [pos_rows][E] (row 0 = CLS,
 * then a square grid*grid table; a non-square count is VA_ERR_INVALID like
 * infer_grid, pos_embed.rs:89-106), register_tokens [num_register][E] (num_register
 * must equal the context's; NULL when 0), interp_offset 0.1 for DA3
 * (DEFAULT_INTERP_OFFSET, pos_embed.rs:41-55).  The filter is stored as bf16.
 *
 * va_prepare_tokens_device = prepare_tokens for `views` images at once: image
 * NCHW F32 [views][3][height][width] -> tokens F32 [views][n][E], n = 1 +
 * num_register + gh*gw, gh = height/patch, gw = width/patch; per view row 0 =
 * cls + pos[0], rows 1..num_register = register tokens, then patch rows
 * (row-major over the patch grid) = conv + bias + pos[1 + p].  position: NULL
 * (the bicubic table of interpolate_pos_embed, pos_embed.rs:122-172, built on
 * the device once per (gh, gw) and cached) or a device table [(1 + gh*gw)][E].
 * height/width not multiples of patch, or views*gh*gw above max_rows, are
 * VA_ERR_INVALID.  Launches only, on `stream`.
 *
 * va_prepare_tokens_host: the same with host buffers (CudaPatchEmbedExecutor::run,
 * patch_embed.rs:200-245, for several views; position NULL or a host table).
 * va_pos_embed_device: the cached interpolated table alone (PosEmbedCache::
 * get_or_build, pos_embed.rs:199-222), out [(1 + gh*gw)][E] on the device. */
int va_load_patch_embed(va_ctx* ctx, const float* weight_oihw, const float* bias,
                        const float* cls_token, const float* pos_embed, int64_t pos_rows,
                        const float* register_tokens, int num_register, int patch,
                        float interp_offset);
int va_prepare_tokens_device(va_ctx* ctx, const float* image, int views, int height, int width,
                             const float* position, float* tokens, void* stream);
int va_prepare_tokens_host(va_ctx* ctx, const float* image, int views, int height, int width,
                           const float* position, float* tokens);
int va_pos_embed_device(va_ctx* ctx, int gh, int gw, float* out, void* stream);

/* Multi-view device route (forward_multi_view_with_persistent_
 * cuda_tail, backbone.rs:885-1137).  va_load_vit_norm uploads vit.norm.weight/bias
 * [E] for the captures.  va_backbone_device runs blocks [first_layer, last_layer)
 * in place on view-major device tokens [view_count * n, E] (n = 1 + num_register +
 * gh*gw): block `layer` is global when alt_start >= 0, layer >= alt_start and layer
 * is odd (backbone.rs:459-460); before block alt_start the camera slots are written
 * into token 0 of every view (view 0 <- slot 0, the others <- slot 1,
 * backbone.rs:746-768; camera_dev [2E] device, or NULL); after the last local block
 * before a global one the tokens are snapshotted on the device.  For each i < n_out
 * with out_layers[i] == layer, after that block: feat_dev[i] [views, n - n_special,
 * W] and cam_dev[i] [views, W] (W = 2E when cat_token, else E) receive the
 * post-processed capture of backbone.rs:1139-1179 (patch rows LayerNormed with
 * vit.norm, concatenated after the local snapshot's rows when cat_token).  Every
 * block needs va_load_layer (with norm1) and va_load_mlp.  Launches only, on
 * `stream`; nothing is copied to the host. */
int va_load_vit_norm(va_ctx* ctx, const float* norm_w, const float* norm_b);
int va_backbone_device(va_ctx* ctx, float* tokens_dev, int64_t rows, int gh, int gw, int view_count,
                       int first_layer, int last_layer, int alt_start, int cat_token,
                       const float* camera_dev, int n_out, const int* out_layers,
                       float* const* feat_dev, float* const* cam_dev, void* stream);
/* The same route over this rank's slice of a window shared by the ranks of a
 * communicator (one process per GPU): tokens_local holds rows [row_offset,
 * row_offset + local_rows) of a window_rows = view_count * n window, whole views
 * (slices may be uneven, e.g. 12 views on 8 GPUs as 2,2,2,2,1,1,1,1).  Local blocks
 * run on the rank's own views with no communication; global blocks exchange K'/V
 * (uneven slices need the direct exchange) and the MLP stays token-local.  The
 * camera slots follow the window's view order (only the rank holding view 0 writes
 * the reference slot); captures cover the rank's own views.  Collective whenever
 * the layer range holds a global block. */
int va_backbone_device_sharded(va_ctx* ctx, float* tokens_local, int64_t local_rows,
                               int64_t row_offset, int64_t window_rows, int gh, int gw,
                               int view_count, int first_layer, int last_layer, int alt_start,
                               int cat_token, const float* camera_dev, int n_out,
                               const int* out_layers, float* const* feat_dev,
                               float* const* cam_dev, void* stream);

/* Multi-GPU (one process per GPU).  The reference has no multi-GPU code; these
 * add the query-sharded global block: each rank owns an equal contiguous slice of
 * the view-major window and forms K'/V for it; the window is then assembled on
 * every rank before the fused attention.  Local blocks need no communication when
 * each rank's slice holds whole views. */
/* Rank 0 creates the 128-byte communicator id and sends it to the other ranks. */
int va_comm_unique_id(void* id_out);
/* Collective.  Creates the NCCL communicator, then maps every peer's key/value
 * window into this process (CUDA IPC, up to 8 ranks).  When every rank mapped
 * every peer, K'/V are exchanged directly (see va_comm_exchange_mode); otherwise,
 * or with VA_KV_EXCHANGE=nccl in every rank's environment, an in-place NCCL
 * all-gather assembles the window. */
int va_comm_init(va_ctx* ctx, const void* id, int nranks, int rank);
/* va_attention_device_sharded with host buffers (pinned for overlap): this rank's
 * ln1_local / out_local F32 [local_rows, E].  The rows are copied in chunks on a
 * copy stream while their LN/QKV (and K'/V exchange stores) run, and the output is
 * copied back chunk by chunk while later attention chunks compute.  Collective. */
int va_attention_host_sharded(va_ctx* ctx, int layer, const float* ln1_local, float* out_local,
                              int64_t local_rows, int gh, int gw, int view_count, int global);
/* 0: no communicator, 1: NCCL all-gather, 2: direct, the QKV epilogue stores each
 * finished K'/V tile into every peer's window over NVLink, then a one-warp kernel
 * raises this rank's flag in every peer (system-scope release, no wait), 3: direct,
 * pushed by copy engines in VA_PUSH_CHUNKS chunks per peer (default: one per 16 MB
 * sent to the peer, at most 4), each chunk
 * followed by a stream memory write of this rank's flag in that peer (one copy
 * stream serving the peers in the order they read this rank's rows, rank - 1 first,
 * or with VA_PUSH_ORDER=parallel one copy stream per peer).
 * A flag holds the call's epoch and how far this rank's rows have arrived.  In modes
 * 2 and 3 the attention kernel starts on the rank's own key tiles and, before each
 * later tile, waits (bounded) only until the rows of that tile are in place.  Where
 * mode 3 is available a call still uses mode 2 when it sends less than 12 MB to each
 * peer (the epilogue stores are faster there).  VA_KV_EXCHANGE=nccl, =sm or =ce at
 * va_comm_init force modes 1, 2 or (where available) 3. */
int va_comm_exchange_mode(const va_ctx* ctx);
/* The path the last sharded call took (codes as above; 0 before any). */
int va_last_exchange(const va_ctx* ctx);
/* ln1_local/out_local: device F32 [local_rows, E], this rank's rows
 * [rank*local_rows, (rank+1)*local_rows) of a window of nranks*local_rows tokens
 * made of view_count views.  Collective: every rank calls it for the same layer. */
int va_attention_device_sharded(va_ctx* ctx, int layer, const float* ln1_local,
                                float* out_local, int64_t local_rows, int gh, int gw,
                                int view_count, int global, void* stream);

/* Kernel-level entry points (each one launch; used by the parity tests). */
/* K2 alone: q bf16 [q_count, heads*64] token-major, k bf16 and v [kv_rows, heads*64];
 * v is bf16 (the production path) or, with v_f16 != 0, f16 (P is then formed in
 * f16).  variant (bf16 path) = poly + 8 * form, or < 0 for the library default
 * (24): poly 0..2 = how many of every 8 exponential pairs run on the FMA pipe
 * instead of MUFU; form 0, 1, 2, 4 = one softmax row per thread (instruction
 * formulations), form 3 = four threads per row (20 warps), form 5 = form 3 with
 * the two query tiles taking turns in the exponential section, form 6 = form 3
 * with the split tail off (one CTA per unit), form 7 = form 3 with P handed over
 * in two 64-key halves, variant 64 = 64-key half-steps with S and P
 * double-buffered in TMEM; with the fixed offset (variant + 256) also form 9..15 +
 * i: keys 0..63+8i of every 128 exponentiated on MUFU and the rest on the FMA pipe by
 * other warps (9: cubic, 10: quadratic, 11/12: the same with the two query tiles
 * taking turns, 13: 10 with a start offset between the tiles, 14: 10 as a persistent
 * walk over the launch's work items, 15: 10 with one query tile per CTA and two CTAs
 * per SM, i = 0..2 only); 511 = the fixed offset with the library's
 * default layout (form 15, i = 1 for local attention and for global launches whose
 * 256-query units fill 1.5 to 2 waves of the SMs; else form 10, i = 1).  variant + 256: exponents relative to 0 instead of
 * the running row max (forms 3 and 9..15; others ignore it), for callers that guarantee
 * |q.k| / 8 * log2(e) <= 64 for every query/key pair (bf16 V only); the layer entry
 * points choose this themselves for QK-normalised layers whose norm weights bound
 * the scores that far (VA_SOFTMAX_FIXED_OFFSET=0 turns it off).  Query i is row
 * q_offset + i of the key window.  seg_len = 0: every query attends to all kv_rows
 * keys; seg_len > 0: independent segments of seg_len tokens (q_offset and q_count
 * multiples of seg_len).  out bf16 [q_count, heads*64]. */
int va_flash_attention_bf16(va_ctx* ctx, const void* q, const void* k, const void* v,
                            int64_t q_count, int64_t q_offset, int64_t kv_rows, int heads,
                            int64_t seg_len, int v_f16, int variant, void* out,
                            void* stream);

/* The launch plan va_flash_attention_bf16 (and every layer entry point) makes for a
 * bf16-V call with these shapes on a GPU of `sms` multiprocessors, with a context's
 * split workspace; host only, needs no GPU.  fixed_offset and variant as above
 * (variant < 0: the library default, + 256: the fixed offset).  plan[9] receives:
 * form, poly, query rows per unit (128 one-tile / 256 two-tile), CTAs per SM the
 * split plan counts, units run whole, key ranges per tail unit (1: no split), and
 * the grid (x, y, z).  VA_ERR_INVALID for shapes or a variant the launch rejects. */
int va_flash_plan(int64_t q_count, int64_t q_offset, int64_t kv_rows, int heads, int64_t seg_len,
                  int fixed_offset, int variant, int sms, int* plan);
/* K3-style GEMM: out[M,N] = (a[M,K] * w_t[N,K]^T + bias) * scale (+ residual), bf16
 * in, F32 out; bias/scale/residual may be NULL.  N % 128 == 0, K % 64 == 0. */
int va_linear_bf16(va_ctx* ctx, const void* a, const void* w_t, const float* bias,
                   const float* scale, const float* residual, float* out, int64_t m, int n, int k,
                   void* stream);

/* Host-side view scheduling (backbone.rs:133-224, engine.rs:198-205). */
/* select_reference_view_saddle: cls [views, embed] F32 -> reference view index. */
int va_select_reference_view_saddle(const float* cls, int views, int embed, int* out_index);
/* reference_first_order: order[0] = reference, then the other views ascending. */
int va_reference_first_order(int views, int reference, int* order_out);
/* restore_original_view_order as a gather: original view i = ordered view src_out[i]. */
int va_restore_order(int views, int reference, int* src_out);
/* Device helpers: camera-token slots (backbone.rs:746-768) and view permutation. */
int va_camera_inject_device(float* tokens_dev, const float* camera_dev, int views,
                            int64_t tokens_per_view, int embed, void* stream);
int va_permute_views_device(const float* src_dev, float* dst_dev, const int* order_host,
                            int views, int64_t view_elems, void* stream);

/* Reads and clears the context's device error word (synchronises the context's
 * device).  Returns VA_OK or VA_ERR_DEVICE with the code in va_last_error. */
int va_check_device(va_ctx* ctx);

/* Phase profile (the reference's DA_PHASE_PROFILE, vit_block.rs:980-990): while
 * enabled, every device-path sub-block call (va_attention_device,
 * va_block_attention_device, va_attention_device_sharded) records CUDA events
 * between its launches.  va_phase_times then returns the last such call's
 * durations in ms, in this order: [0] ln (LN1 / bf16 cast), [1] qkv (QKV GEMM with
 * the fused qk_norm_rope and head pack), [2] all-gather of K'/V (0 unless sharded),
 * [3] core (flash attention, unpack fused), [4] proj.  Profiling adds no
 * synchronisation to the call; va_phase_times waits for the last event. */
int va_set_phase_profile(va_ctx* ctx, int enable);
int va_phase_times(va_ctx* ctx, float* ms_out /* [5] */);
/* With the phase profile enabled: the copy-engine K'/V push of the last profiled
 * sharded call, per peer (no reference counterpart; the reference has no
 * multi-GPU path): ms_out[p] = time from the first copy to this peer to its last
 * flag (CUDA events on the copy stream), *npeer_out peers, *bytes_per_peer bytes
 * (this rank's K' and V rows) sent to each; *npeer_out = 0 when the last profiled
 * call pushed nothing by copy engines.  VA_ERR_STATE before any profiled call. */
int va_exchange_times(va_ctx* ctx, float* ms_out /* [7] */, int* npeer_out, int64_t* bytes_per_peer);

/* Failure-detection self-test (no reference counterpart; the reference has no
 * device-side waits).  Launches one kernel whose only wait is on a barrier that
 * nothing arrives on, through the same bounded wait the attention kernels use,
 * with a limit of limit_us microseconds (1 .. 1e6).  The wait gives up, the
 * kernel writes a timeout code into the device error word and returns; the call
 * then returns VA_ERR_DEVICE exactly as a stalled attention launch would, and the
 * context stays usable.  Any other status means the mechanism is broken. */
int va_selftest_bounded_wait(va_ctx* ctx, int64_t limit_us);
/* Self-test of the attention kernel's wait for peer rows (the copy-engine K'/V
 * exchange) on one GPU: a 1-head, 256-key launch as rank 0 of 2 owning the first
 * 128 keys; peer_flag != 0 raises rank 1's flag (epoch 1, all rows in place).  peer_flag != 0:
 * VA_OK and *out_max_abs = max |difference| to the same launch without a peer
 * (0: same key order).  peer_flag 0: the kernel gives up after its 2 s wait limit
 * and the call returns VA_ERR_DEVICE; the context stays usable. */
int va_selftest_peer_wait(va_ctx* ctx, int peer_flag, float* out_max_abs);

/* ------------------------------------------------------------------ GGUF model files
 * The reference's crates/da-gguf reader (reader.rs, meta.rs, q8_0.rs), ModelConfig::
 * from_gguf (config.rs:219-264) and weights_from_gguf (engine.rs:110-126).  The
 * reader parses a read-only mapping of the file on the host; tensor data is
 * converted to F32 / bf16 on the GPU.  Messages of failing va_gguf_* calls are in
 * va_gguf_last_error() (per thread), worded like the reference's GgufError. */
typedef struct va_gguf va_gguf;

/* Kinds of metadata values, the MetaValue variants (meta.rs:1-12).  uint8/uint16
 * keys read as U32, int8/int16 as I32 (an int8 byte zero-extended, as the reference
 * does), int64 as U64 (bit pattern), float64 as F32; arrays of other element types
 * are skipped and not listed. */
#define VA_META_U32 0
#define VA_META_I32 1
#define VA_META_F32 2
#define VA_META_U64 3
#define VA_META_BOOL 4
#define VA_META_STR 5
#define VA_META_ARR_U32 6
#define VA_META_ARR_I32 7
#define VA_META_ARR_F32 8
#define VA_META_ARR_STR 9

/* GGML tensor types the reader converts (reader.rs:52-55). */
#define VA_GGML_F32 0
#define VA_GGML_F16 1
#define VA_GGML_Q8_0 8

/* GgufFile::open (reader.rs:213-266): versions 2 and 3, `general.alignment` (u32)
 * or 32.  VA_ERR_IO, VA_ERR_FORMAT ("bad magic", "unsupported gguf version N",
 * "malformed: ...").  The mapping lives until va_gguf_close. */
int va_gguf_open(const char* path, va_gguf** out);
void va_gguf_close(va_gguf* g);
const char* va_gguf_last_error(void);
int va_gguf_version(const va_gguf* g, uint32_t* version);

/* Metadata in file order; a key that occurs twice answers with its first entry
 * (meta.rs:16-18).  Keys and names are looked up as NUL-terminated strings; the
 * enumerators also give their byte length (a key may hold a NUL byte, which makes
 * it reachable by enumeration only).  Getters coerce like meta.rs: u32 accepts I32 (bit cast), i32
 * accepts U32, arr_i32 accepts ARR_U32; otherwise an absent key or another kind is
 * VA_ERR_NOT_FOUND (the reference's None).  Strings stay owned by the file handle.
 * Array getters copy min(count, cap) values and return VA_ERR_CAPACITY when cap <
 * count (out may be NULL to query the count). */
int va_gguf_meta_count(const va_gguf* g, int64_t* n);
int va_gguf_meta_entry(const va_gguf* g, int64_t i, const char** key, int64_t* key_len, int* kind);
int va_gguf_meta_u32(const va_gguf* g, const char* key, uint32_t* out);
int va_gguf_meta_i32(const va_gguf* g, const char* key, int32_t* out);
int va_gguf_meta_f32(const va_gguf* g, const char* key, float* out);
int va_gguf_meta_u64(const va_gguf* g, const char* key, uint64_t* out);
int va_gguf_meta_bool(const va_gguf* g, const char* key, int* out);
int va_gguf_meta_str(const va_gguf* g, const char* key, const char** s, int64_t* len);
int va_gguf_meta_arr_u32(const va_gguf* g, const char* key, uint32_t* out, int64_t cap, int64_t* count);
int va_gguf_meta_arr_i32(const va_gguf* g, const char* key, int32_t* out, int64_t cap, int64_t* count);
int va_gguf_meta_arr_f32(const va_gguf* g, const char* key, float* out, int64_t cap, int64_t* count);
/* Element i of a string array (s/len may be NULL to query only the count). */
int va_gguf_meta_arr_str(const va_gguf* g, const char* key, int64_t i, const char** s, int64_t* len,
                         int64_t* count);

/* Tensors in file order (tensor_names, meta.rs:90-92).  shape is outer -> inner
 * (stored dims reversed, reader.rs:300); VA_ERR_CAPACITY when shape_cap < ndims. */
int va_gguf_tensor_count(const va_gguf* g, int64_t* n);
int va_gguf_tensor_name(const va_gguf* g, int64_t i, const char** name, int64_t* name_len);
int va_gguf_tensor_info(const va_gguf* g, const char* name, int* dtype, int* ndims, int64_t* shape,
                        int shape_cap, uint64_t* offset);
/* The checks of tensor_f32 / tensor_q8_0 (reader.rs:279-376), in their order:
 * VA_ERR_NOT_FOUND "tensor not found: X"; Q8_0 element count not a multiple of 32
 * and data past the end of the file: VA_ERR_FORMAT; other types: VA_ERR_DTYPE.
 * On success: element count and the stored bytes inside the mapping (a Q8_0 tensor's
 * 34-byte blocks, tensor_q8_0's view). */
int va_gguf_tensor_check(const va_gguf* g, const char* name, int64_t* numel, const void** data,
                         int64_t* nbytes);
/* tensor_f32 on the GPU: the tensor's F32 values into out (device, numel floats);
 * with transpose2d a rank-2 [rows, cols] tensor comes out [cols, rows], as
 * weights_from_gguf stores it.  Runs on `stream` of the current device and returns
 * when the values are written.  Q8_0 and F16 values are exact in F32, so the result
 * equals the reference's host decoding bit for bit. */
int va_gguf_tensor_device(const va_gguf* g, const char* name, int transpose2d, float* out, void* stream);
/* The same conversion with the values copied back to host memory (out holds cap
 * floats; VA_ERR_CAPACITY when the tensor has more): tensor_f32's result, computed
 * on the current device.  Synchronous. */
int va_gguf_tensor_f32(const va_gguf* g, const char* name, int transpose2d, float* out, int64_t cap);

/* ModelConfig (config.rs:146-...) as read by ModelConfig::from_gguf: arch must be
 * "depthanything3" (else VA_ERR_INVALID), required keys missing or of another kind
 * are VA_ERR_NOT_FOUND "missing required gguf metadata key: K" (first in the
 * struct's order), img.mean/img.std of a length other than 3 are VA_ERR_FORMAT;
 * defaults: ffn_type "mlp", alt_start -1, cat_token 1, head_max_depth 0,
 * head_pos_embed 1; image_size from img.resize_target, else image_size. */
#define VA_MAX_OUT_LAYERS 16
typedef struct va_model_config {
  char arch[32];
  uint32_t patch_size, image_size, embed_dim, depth, num_heads, head_dim, mlp_hidden, num_register;
  int32_t rope_start, qknorm_start;
  float rope_freq, ln_eps;
  int32_t out_layers[VA_MAX_OUT_LAYERS];
  int32_t n_out_layers;
  char ffn_type[16];
  int32_t alt_start, cat_token;
  uint32_t head_features;
  float head_max_depth;
  int32_t head_pos_embed;
  float img_mean[3], img_std[3];
  char img_resize_mode[32];
  uint32_t cam_dim_in;
} va_model_config;
int va_gguf_model_config(const va_gguf* g, va_model_config* cfg);

/* weights_from_gguf + every va_load_* of the context in one pass, without host F32
 * copies: each tensor's stored bytes go to the GPU (two pinned staging buffers) and
 * one kernel writes the context's operand directly (F32 vectors; bf16 K-major
 * matrices, where a rank-2 tensor's GGUF order [out, in] already is the operand
 * and a flat tensor, which the reference reads as [in, out], is transposed).  For
 * each block i < depth with vit.blk.{i}.attn_qkv.weight: the va_load_layer set
 * (norm1, attn_qkv, attn_qnorm/knorm, attn_proj, ls1; absent optional tensors as
 * NULL), and with vit.blk.{i}.mlp_fc1.weight the va_load_mlp set; with
 * vit.patch_embed.weight the va_load_patch_embed set (patch_embed weight/bias,
 * cls_token, pos_embed, register_tokens when num_register > 0); vit.norm.* when
 * present.  Shapes are checked against the context (VA_ERR_INVALID); GGUF errors as
 * above with the message in va_last_error.  *uploaded_bytes (optional) = stored
 * bytes sent.  Synchronous. */
int va_load_model_gguf(va_ctx* ctx, const va_gguf* g, int64_t* uploaded_bytes);

#ifdef __cplusplus
}
#endif

#endif /* VESTRA_ATTN_H */
