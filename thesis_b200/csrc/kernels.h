// Internal launchers of the non-GEMM kernels (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace eesd {

struct AttnGeom {
  int n_heads, n_kv_heads, head_dim;
  int max_batch, max_seq;
  int ld_q;          // elements between consecutive tokens' q rows (the fused qkv row)
  float scale;       // 1 / sqrt(head_dim)
  int n_tokens, n_blocks;   // of the packed batch: items and blocks are checked against them
  uint32_t spin;     // poll limit of the key-tile waits (spin_limit())
  int* status;       // device status word (fp32 kernel; the bf16 kernel takes it as an argument)
  int n_items = 0;                  // work items of the launch (set by launch_attention)
  const int32_t* order = nullptr;   // bf16 kernel: item of each grid slot (launch_attn_order), or identity
};

int attn_item_tokens(int n_heads, int n_kv_heads);
// record the text eesd_last_error() returns for the calling thread
void set_last_error(const char* msg);

// rows (nullable): source row of each output row, checked against [0, n_src) (a bad one sets
// kStatusBadIndex in *status and zeroes its output row)
int launch_rmsnorm(int dtype, const void* x, const int32_t* rows, const void* w, void* y, int n, int dim, float eps,
                   cudaStream_t s, int n_src = 0x7fffffff, int* status = nullptr);
int launch_rope_kv(int dtype, void* qkv, const int32_t* tok_pos, const int32_t* tok_row, int n_tok, int n_heads,
                   int n_kv_heads, int head_dim, const float* cos, const float* sin, void* kc, void* vc, int max_batch,
                   int max_seq, int* status, cudaStream_t s);
// RoPE + KV append done by the bf16 attention kernel itself (every block of the batch must fit
// one work item, so the CTA that appends a block's keys is the only one that reads them):
// q, k, v are read unrotated from the fused projection, q rotated in shared memory, k rotated
// and v copied into this layer's caches kc / vc ([max_batch, Hkv, max_seq, D]).
struct AttnAppend {
  bool on = false;
  void* kc = nullptr;
  void* vc = nullptr;
  const float* cos = nullptr;   // [max_seq, D]
  const float* sin = nullptr;
};
// kc / vc: the whole cache [n_layers, max_batch, Hkv, max_seq, D]; bf16 reads it through the
// 2-D TMA maps kmap / vmap ([n_layers * max_batch * Hkv * max_seq, D], 64 x 64 boxes, 128B swizzle)
int launch_attention(int dtype, const AttnGeom& g, const void* q, const void* kc, const void* vc, void* out,
                     const int32_t* blk, const int32_t* items, int n_items, int max_ctx, int* status, cudaStream_t s,
                     const CUtensorMap* kmap, const CUtensorMap* vmap, int layer, const AttnAppend& app = AttnAppend(),
                     int rows_max = 32);   // rows_max: largest item's query rows (tokens x GQA group)
// order[j] = the item the bf16 attention grid runs j-th: items by descending key count (ties by
// index), so the longest start in the first wave.  At most kAttnOrderMax items.
constexpr int kAttnOrderMax = 4096;
int launch_attn_order(const int32_t* blk, const int32_t* items, int n_items, int n_blocks, int n_heads, int n_kv_heads,
                      int32_t* order, cudaStream_t s);
int launch_embed(int dtype, const void* table, const int32_t* ids, int n, int dim, int vocab, void* x, int* status,
                 cudaStream_t s);
int launch_copy_rows(int dtype, const void* src, const int32_t* src_idx, void* dst, const int32_t* dst_idx, int n,
                     int width, cudaStream_t s);
int launch_gather_ids(const int32_t* table, const int32_t* idx, int32_t* ids, int n, cudaStream_t s);
int launch_scatter_ids(const int32_t* ids, const int32_t* idx, int32_t* table, int n, cudaStream_t s);
int launch_greedy_accept(const int32_t* y, const int32_t* vinfo, int nv, int32_t* seq_buf, int stride, int32_t* acc,
                         cudaStream_t s);
int launch_round_meta(const int32_t* act, int n, const int32_t* pos, int max_batch, int cols, int item_tokens,
                      int32_t* out, cudaStream_t s);
int launch_round_advance(const int32_t* act, int n, const int32_t* acc, int32_t* pos, int max_batch, cudaStream_t s);
// status (nullable): a non-zero word makes every id -1; status_out (nullable) receives the word
int launch_keys_to_ids(const unsigned long long* keys, int32_t* ids, int n, cudaStream_t s,
                       const int* status = nullptr, int32_t* status_out = nullptr);
int launch_argmax_rows(int dtype, const void* logits, int n, int vocab, int32_t* ids, cudaStream_t s);
int launch_swiglu_f32(const float* gu, float* out, int n, int inter, cudaStream_t s);
int launch_simt_gemm_f32(int epi, const float* x, const float* w, const float* residual, float* y, int n_tok, int n_out,
                         int k, cudaStream_t s);

}  // namespace eesd
