/*
 * eesd.h — C ABI of the B200 (sm_100a) kernels for the packed, ragged LayerSkip-Llama
 * draft/verify step.
 *
 * Conventions
 *   - Every pointer argument is a DEVICE pointer unless marked "host".
 *   - `stream` is a cudaStream_t passed as void*.  Nothing here synchronises the stream,
 *     allocates device memory or frees it: the caller owns every buffer.
 *   - Every function returns an int status (EESD_OK = 0).  Argument errors are detected on
 *     the host before any launch; device-side faults of the data (an out-of-range row,
 *     position or token id) and bounded-wait timeouts are OR-ed into a device status word
 *     that eesd_model_check() / eesd_status_read() return.
 *   - Element types: EESD_BF16 or EESD_F32 (the model dtype; tcgen05 GEMMs serve bf16, a
 *     CUDA-core FFMA GEMM serves the fp32 parity path).
 *   - Token ids, positions and cache rows are int32.
 *
 * Packed batch (the reference's `PackedBatch`, solutions/packed.py:63-78): tokens of
 * several request blocks are concatenated on one axis; block b holds T_b consecutive
 * tokens at positions pos0_b .. pos0_b+T_b-1 of KV-cache row row_b.  A query at position
 * p of row r attends to cached positions <= p of row r after this call's K/V are written
 * (solutions/packed.py:6-8).
 */
#ifndef EESD_H
#define EESD_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EESD_OK 0
#define EESD_ERR_ARG 1         /* invalid argument or unsupported shape (nothing launched)  */
#define EESD_ERR_CUDA 2        /* a CUDA runtime / driver call failed                       */
#define EESD_ERR_DEVICE 3      /* the device status word is non-zero (see eesd_status_*)    */

#define EESD_BF16 0
#define EESD_F32 1

/* GEMM epilogues (y[t, o] for token t, output feature o) */
#define EESD_EPI_STORE 0       /* y = acc                                                   */
#define EESD_EPI_RESIDUAL 1    /* y = residual + round(acc)   (x + F.linear(...))           */
#define EESD_EPI_SWIGLU 2      /* y = silu(round(g)) * round(u), g/u = rows o and o+up_offset */

/* Launch categories for the optional per-kernel CUDA-event profile */
#define EESD_PROF_NORM 0
#define EESD_PROF_GEMM_QKV 1
#define EESD_PROF_ROPE_KV 2
#define EESD_PROF_ATTN 3
#define EESD_PROF_GEMM_O 4
#define EESD_PROF_GEMM_W13 5
#define EESD_PROF_GEMM_W2 6
#define EESD_PROF_HEAD 7
#define EESD_PROF_MISC 8
#define EESD_PROF_KINDS 9

/* Library version and the text of the last host-side error of the calling thread. */
int eesd_version(void);
const char* eesd_last_error(void);

/* ------------------------------------------------------------------------------------ */
/* Model runtime.  Replaces the weight/KV layout of LayerSkipLlama (common/model.py:161-183,
 * 222-293) and the per-layer loop of packed_layers (solutions/packed.py:169-196).        */

typedef struct EesdModelDesc {
  int32_t dtype;                 /* EESD_BF16 | EESD_F32 */
  int32_t n_layers, dim, n_heads, n_kv_heads, head_dim, intermediate, vocab;
  float norm_eps;
  int32_t max_batch;             /* KV-cache rows */
  int32_t max_seq;               /* positions per row (multiple of 64) */
  int32_t max_tokens;            /* largest packed token count of one call */
  int32_t weights_packed;        /* bf16 only: 1 = wqkv, wo, w13, w2 and lm_head point to tile-packed
                                    copies (eesd_pack_weight), read as contiguous 16 KB tiles */
  /* per-layer weights: arrays (host memory) of n_layers device pointers */
  const void* const* wqkv;       /* [(Hq + 2 Hkv) D, dim] rows = [q; k; v] (common/model.py:262-263) */
  const void* const* wo;         /* [dim, Hq D] */
  const void* const* w13;        /* [2 I, dim] rows = [gate; up] (common/model.py:264-265) */
  const void* const* w2;         /* [dim, I] */
  const void* const* attn_norm;  /* [dim] */
  const void* const* ffn_norm;   /* [dim] */
  const void* final_norm;        /* [dim] */
  const void* lm_head;           /* [vocab, dim] (the embedding when tied) */
  const void* embed;             /* [vocab, dim] */
  const float* rope_cos;         /* [max_seq, D] fp32, rotate-half layout (common/model.py:129-140) */
  const float* rope_sin;
  void* k_cache;                 /* [n_layers, max_batch, Hkv, max_seq, D] (common/model.py:171-179) */
  void* v_cache;
  void* workspace;               /* eesd_model_workspace_bytes() bytes, 256-byte aligned */
  size_t workspace_bytes;
} EesdModelDesc;

/* One packed call (PackedBatch, solutions/packed.py:63-139, minus buckets and masks). */
typedef struct EesdBatch {
  int32_t n_tokens;
  int32_t n_blocks;
  int32_t n_items;               /* attention work items (block, query tile) */
  int32_t max_ctx;               /* host: max over blocks of pos0 + T */
  const int32_t* tok_pos;        /* [n_tokens] absolute position of every token */
  const int32_t* tok_row;        /* [n_tokens] KV-cache row of every token */
  const int32_t* blk;            /* [n_blocks, 4] = (start, T, row, pos0) */
  const int32_t* items;          /* [n_items, 2] = (block, first token within block) */
} EesdBatch;

/* Tile-packed weight layout for the bf16 GEMMs: a [rows, k] row-major bf16 matrix (k % 64 == 0)
 * becomes [ceil(rows/128) * k/64][128][64]: the 128 x 64 operand tile (row tile m, k-block j) is
 * the contiguous 16 KB block m * (k/64) + j, so each CTA streams its weights sequentially from HBM
 * (rows past the end are zero).  Layout change only; the GEMM numerics are unchanged.  w13 needs
 * intermediate % 128 == 0 to be packed as one matrix. */
size_t eesd_packed_weight_bytes(int rows, int k);
int eesd_pack_weight(const void* w, int rows, int k, void* out, void* stream);

/* Query tokens per attention work item for a model (items tile every block by this). */
int eesd_attn_item_tokens(int n_heads, int n_kv_heads);

size_t eesd_model_workspace_bytes(const EesdModelDesc* desc);
int eesd_model_create(const EesdModelDesc* desc, void** handle_out);
int eesd_model_destroy(void* handle);

/* Layers [start, end) on the packed hidden states x [n_tokens, dim] (in place), writing this
 * call's K/V into the cache.  solutions/packed.py:169-196 (packed_layer / packed_layers). */
int eesd_forward_layers(void* handle, void* x, const EesdBatch* batch, int start, int end, void* stream);

/* Shared exit head: final RMSNorm + LM head + greedy argmax over rows `rows` (nullable =
 * 0..n-1) of x.  common/model.py:328-330 with solutions/engine.py:352,463 (argmax).
 * out_ids [n] int32; logits (nullable) [n, vocab] in the model dtype. */
int eesd_head_argmax(void* handle, const void* x, const int32_t* rows, int n, int32_t* out_ids, void* logits,
                     void* stream);

/* x[i] = embed[ids[i]] (common/model.py:325-326), ids [n] int32. */
int eesd_embed(void* handle, const int32_t* ids, int n, void* x, void* stream);

/* Copy the device status word of the model to the host (synchronous on `stream`) and clear
 * it.  Returns EESD_ERR_DEVICE when any bit was set; *bits_out (host, nullable) gets them. */
int eesd_model_check(void* handle, int* bits_out, void* stream);

/* Per-kernel CUDA-event timing of the runtime's launches (off by default).  enable=1 starts a
 * new window; read fills ms[EESD_PROF_KINDS] and launches[EESD_PROF_KINDS] (host arrays) after
 * synchronising the recorded events. */
int eesd_model_profile(void* handle, int enable);
int eesd_model_profile_read(void* handle, double* ms, int64_t* launches);

/* The recorded launches one by one (kind, packed token count, ms), at most `cap` (host
 * arrays, each nullable); returns the number written, or -1 on error. */
int eesd_model_profile_records(void* handle, int32_t* kinds, int32_t* n_tok, float* ms, int cap);

/* Number of kernel launches the runtime issued since creation (host counter). */
int64_t eesd_model_launch_count(void* handle);

/* ------------------------------------------------------------------------------------ */
/* Step kernels of the EESD engine.  solutions/engine.py:345-352, 453-475.              */

/* dst[i, :] = src[src_idx[i], :] (src_idx nullable = i); dst_idx (nullable = i) scatters. */
int eesd_copy_rows(int dtype, const void* src, const int32_t* src_idx, void* dst, const int32_t* dst_idx, int n,
                   int width, void* stream);

/* ids[i] = table[idx[i]] (int32 gather, e.g. input ids from the token buffer seq_buf). */
int eesd_gather_ids(const int32_t* table, const int32_t* idx, int32_t* ids, int n, void* stream);

/* ids scatter: table[idx[i]] = ids[i] (e.g. drafts into seq_buf). */
int eesd_scatter_ids(const int32_t* ids, const int32_t* idx, int32_t* table, int n, void* stream);

/* Greedy acceptance (solutions/engine.py:464-475; common/engine.py:386-388).  For verifier v
 * with vinfo[v] = (start, T, slot): the verified tokens are y[start .. start+T-1] and the
 * drafts are seq_buf[slot * stride + 1 .. T-1].  acc[v] = first j < T-1 with
 * y[start+j] != draft j (else T-1); seq_buf[slot * stride] = y[start + acc[v]]. */
int eesd_greedy_accept(const int32_t* y, const int32_t* vinfo, int nv, int32_t* seq_buf, int stride, int32_t* acc,
                       void* stream);

/* Device-built metadata of one synchronous draft/verify round (gamma drafts + 1 verify), so the
 * host can enqueue round r+1 before it reads round r's acceptance (the reference's host packing,
 * solutions/packed.py:81-139, and position update, solutions/engine.py:373-396, done on the GPU).
 * act [n]: the round's cache rows; pos [max_batch]: round-start position per row.  out holds
 * eesd_round_meta_ints(n, gamma, item_tokens) int32, cols = gamma + 1, ni = ceil(cols/item_tokens):
 *   shallow step j = 0..cols-1 at j * 10 n: tok_pos [n] = pos + j, tok_row [n], blk [n, 4] =
 *     (i, 1, row, pos + j), items [n, 2] = (i, 0), src [n] = row * cols + j, dst [n] = src + 1
 *   verify at cols * 10 n: tok_pos [n cols], tok_row [n cols], blk [n, 4] = (i cols, cols, row,
 *     pos), items [n ni, 2], rows [n cols] = row * cols + t, vinfo [n, 3] = (i cols, cols, row)
 * eesd_round_advance: pos[act[i]] += acc[i] + 1 (rollback by length, solutions/engine.py:12-14). */
size_t eesd_round_meta_ints(int n, int gamma, int item_tokens);
int eesd_round_meta(const int32_t* act, int n, const int32_t* pos, int max_batch, int gamma, int item_tokens,
                    int32_t* out, void* stream);
int eesd_round_advance(const int32_t* act, int n, const int32_t* acc, int32_t* pos, int max_batch, void* stream);

/* ------------------------------------------------------------------------------------ */
/* Primitive kernels (exported for tests and for callers composing their own step).    */

/* y[i] = rms_norm(x[rows ? rows[i] : i]) * w   (common/model.py:153-156) */
int eesd_rmsnorm(int dtype, const void* x, const int32_t* rows, const void* w, void* y, int n, int dim, float eps,
                 void* stream);

/* Varlen GQA attention of one packed batch over ONE layer's KV cache.  solutions/packed.py:142-166
 * (`_attend`: per-bucket SDPA over [b, Hkv, G T, D] queries with a bool mask) without buckets or
 * masks: query (token t of block b, head h) attends to positions <= pos0_b + t of row row_b.
 * qkv [n_tokens, (Hq + 2 Hkv) D] is the fused projection output (q heads first, then k, then v);
 * k_cache / v_cache [max_batch, Hkv, max_seq, D]; out [n_tokens, Hq D].  The batch's `items` tile
 * every block into work items of eesd_attn_item_tokens() tokens (tok_pos / tok_row are unused).
 * append = 0: q is used as given (already rotated) and the cache already holds this call's keys.
 * append = 1 (bf16, every block one item, no two blocks on the same cache row): the kernel applies
 * RoPE (rope_cos / rope_sin [max_seq, D] fp32, solutions/packed.py:176-177) to q and k and writes k,
 * v at (row, position) first (solutions/packed.py:180-181).  Each work item appends only its own
 * block's keys, so a row's blocks must come in separate calls (or use eesd_rope_kv_append first).  An item whose block lies outside the batch or whose positions lie
 * outside its row sets a bit in *status (device int32, nullable) and is skipped. */
int eesd_attn_varlen_gqa(int dtype, const void* qkv, int n_heads, int n_kv_heads, int head_dim, void* k_cache,
                         void* v_cache, int max_batch, int max_seq, const EesdBatch* batch, int append,
                         const float* rope_cos, const float* rope_sin, void* out, int32_t* status, void* stream);

/* RoPE of q and k and the in-place KV append of a packed batch (common/model.py:143-150 apply_rope,
 * solutions/packed.py:176-181): q rotated in place in qkv, rotated k and v written to
 * k_cache / v_cache [max_batch, Hkv, max_seq, D] at (tok_row[t], tok_pos[t]).  A token whose row or
 * position is out of range sets a bit in *status (nullable) and is skipped. */
int eesd_rope_kv_append(int dtype, void* qkv, const int32_t* tok_pos, const int32_t* tok_row, int n_tok, int n_heads,
                        int n_kv_heads, int head_dim, const float* rope_cos, const float* rope_sin, void* k_cache,
                        void* v_cache, int max_batch, int max_seq, int32_t* status, void* stream);

/* y[n_tok, n_out] = epilogue(x[n_tok, k] @ w[n_out(+up), k]^T).  workspace: see
 * eesd_gemm_workspace_bytes (split-K partials and tile counters; zeroed by this call). */
size_t eesd_gemm_workspace_bytes(int n_tok, int n_out, int k, int epilogue);
int eesd_gemm(int dtype, int epilogue, const void* x, const void* w, const void* residual, void* y, int n_tok,
              int n_out, int k, int up_offset, void* workspace, size_t workspace_bytes, void* stream);

/* Tuning knobs.  EESD_OPT_MMA_N: N of one tcgen05.mma in the bf16 GEMM (0 = the whole token
 * tile, else a fixed multiple of 16 up to 256); numerics-neutral by design.  EESD_OPT_SPLITS:
 * split-K count (0 = derived from the weight shape; any fixed value keeps batch invariance but
 * changes the summation order, so AR and speculative runs must use the same value).
 * EESD_OPT_STAGES: TMA pipeline depth (0 = as many stages as fit; numerics-neutral).
 * EESD_OPT_PAIR: 1 (default) runs SwiGLU GEMMs on CTA pairs (cta_group::2, M = 256) where the
 * weight shape allows, 0 on single CTAs; AR and speculative runs must use the same value.
 * EESD_OPT_HEAD_TWO_TILES: 1 (default) lets an LM-head launch of up to 256 tokens take two
 * 128-row tiles per CTA (two accumulators), 0 one; numerics-neutral. */
#define EESD_OPT_MMA_N 1
#define EESD_OPT_SPLITS 2
#define EESD_OPT_STAGES 3
#define EESD_OPT_PAIR 4
#define EESD_OPT_HEAD_TWO_TILES 5
/* EESD_OPT_SPIN_LIMIT (tests of the failure path): poll limit of the pipeline waits of the GEMM and
 * attention kernels launched afterwards; -1 restores the default (2^24 polls), 0 makes every such
 * wait give up at once.  A wait that gives up sets a timeout bit in the device status word, the
 * kernel lets the copies and MMAs it already issued land, and returns. */
#define EESD_OPT_SPIN_LIMIT 6
/* EESD_OPT_MMA_SPLIT: a bf16 GEMM token tile above 256 tokens on one CTA takes two MMAs per K16
 * step; this sets the first one's N (a multiple of 16, default 192), the second takes the rest.
 * 0 = two equal halves.  Numerics-neutral. */
#define EESD_OPT_MMA_SPLIT 7
int eesd_set_option(int option, int value);

/* Exit head that allocates nothing, for callers that cannot call cudaMalloc (a serving
 * runtime whose allocator is locked on its decode path, code inside a foreign stream capture, a
 * plug-in that only receives input/output pointers).  No counterpart in the reference: it is the
 * same computation as eesd_head_argmax (final RMSNorm with norm_w, LM head, greedy argmax of rows
 * `rows` (nullable = 0..n-1) of x [x_rows, dim] bf16 -> out_ids [n] int32) without a model handle
 * or workspace.  Its scratch is a fixed 2 MiB + 1280 B __device__ array inside the library, held
 * by every GPU that loads the library until exit.  Limits: bf16, 1 <= n <= 128, dim a multiple of
 * 64 up to 8192; larger sizes return EESD_ERR_ARG with a message.  `stream` must belong to the
 * current device.  The first call on a device resolves the array's device address
 * (cudaGetSymbolAddress) and should come before any stream capture.  All calls share the array:
 * calls that overlap on the GPU race and must be serialised by the caller.
 * Device-side errors: a row index outside [0, x_rows) or a bounded wait that gave up makes every
 * out_id -1, and the call's status bits (0 = none) are written to *status_out (device int32,
 * nullable), both on the stream. */
int eesd_head_argmax_static(const void* x, int x_rows, const int32_t* rows, int n, int dim, int vocab,
                            const void* norm_w, const void* lm_head, float eps, int32_t* out_ids,
                            int32_t* status_out, void* stream);

/* Device status word helpers for the primitive kernels (a caller-owned int32). */
int eesd_status_read(const int32_t* status, int* bits_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* EESD_H */
