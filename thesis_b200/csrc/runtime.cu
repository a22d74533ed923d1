// Native runtime behind the C ABI (include/eesd.h): model handle with pre-encoded TMA
// descriptors for every weight, a caller-provided workspace carved into the activation and
// scratch buffers, the layer-range driver (solutions/packed.py:169-196), the shared exit head
// with fused argmax (common/model.py:328-330), and an optional per-kernel CUDA-event profile.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "common.cuh"
#include "gemm_tc.h"
#include "kernels.h"

#define EESD_VERSION 100

namespace eesd {
namespace {

thread_local std::string g_err;
uint32_t g_spin_limit = kSpinLimit;   // pipeline-wait poll limit (EESD_OPT_SPIN_LIMIT)

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(EESD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

struct Carve {
  size_t off = 0;
  size_t take(size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  }
};

struct ProfEvent {
  int kind;
  int n_tok;
  cudaEvent_t a, b;
};

struct Model {
  EesdModelDesc d;
  int eb;                       // element bytes
  int qkv_dim, q_dim;
  std::vector<const void*> wqkv, wo, w13, w2, attn_norm, ffn_norm;
  std::vector<CUtensorMap> map_qkv, map_o, map_13, map_2;
  CUtensorMap map_head;
  CUtensorMap map_kc, map_vc;   // whole KV cache as [layers * rows * Hkv * max_seq, D], 64 x 64 boxes
  // workspace pieces
  int* status;
  void *xn, *qkv, *attn, *act;
  int32_t* attn_order;          // bf16 attention: item of each grid slot, longest first
  float* gu;                    // fp32 path: [max_tokens, 2 I]
  float* logits32;              // fp32 path: [kHeadChunk, vocab]
  unsigned long long* keys;
  TcScratch gemm_scratch;       // split-K partial tiles of the bf16 GEMM
  int64_t launches = 0;
  bool prof = false;
  std::vector<ProfEvent> events;
  std::vector<cudaEvent_t> pool;
  size_t pool_used = 0;
};

constexpr int kHeadChunk = 128;

struct Layout {
  size_t status, xn, qkv, attn, act, gu, logits32, keys, order, partials, partial_bytes, total;
};

Layout layout_for(const EesdModelDesc& d) {
  Layout L{};
  const int eb = d.dtype == EESD_BF16 ? 2 : 4;
  const size_t T = (size_t)d.max_tokens;
  const int q_dim = d.n_heads * d.head_dim, qkv_dim = (d.n_heads + 2 * d.n_kv_heads) * d.head_dim;
  Carve c;
  L.status = c.take(256);
  L.xn = c.take(T * d.dim * eb);
  L.qkv = c.take(T * qkv_dim * eb);
  L.attn = c.take(T * q_dim * eb);
  L.act = c.take(T * d.intermediate * eb);
  L.gu = c.take(d.dtype == EESD_F32 ? T * 2 * d.intermediate * 4 : 0);
  L.logits32 = c.take(d.dtype == EESD_F32 ? (size_t)kHeadChunk * d.vocab * 4 : 0);
  L.keys = c.take(T * 8);
  L.order = c.take((size_t)kAttnOrderMax * 4);
  if (d.dtype == EESD_BF16) {
    // split-K scratch that covers every projection at up to max_tokens tokens (the LM head is
    // never split)
    const int shapes[4][3] = {{qkv_dim, d.dim, EESD_EPI_STORE},
                              {d.dim, q_dim, EESD_EPI_RESIDUAL},
                              {d.intermediate, d.dim, EESD_EPI_SWIGLU},
                              {d.dim, d.intermediate, EESD_EPI_RESIDUAL}};
    for (const auto& sh : shapes)
      L.partial_bytes = std::max(L.partial_bytes, tc_partial_bytes_max((int)T, sh[0], sh[1], sh[2]));
  }
  L.partials = c.take(L.partial_bytes);
  L.total = c.off;
  return L;
}

void prof_begin(Model* m, cudaStream_t s, int kind, ProfEvent* pe, int n_tok = 0) {
  if (!m->prof) return;
  if (m->pool_used + 2 > m->pool.size()) {
    for (int i = 0; i < 64; ++i) {
      cudaEvent_t e;
      cudaEventCreate(&e);
      m->pool.push_back(e);
    }
  }
  pe->kind = kind;
  pe->n_tok = n_tok;
  pe->a = m->pool[m->pool_used++];
  pe->b = m->pool[m->pool_used++];
  cudaEventRecord(pe->a, s);
}
void prof_end(Model* m, cudaStream_t s, ProfEvent* pe) {
  if (!m->prof) return;
  cudaEventRecord(pe->b, s);
  m->events.push_back(*pe);
}

// GEMM on the packed tokens with one of the model's pre-encoded weight maps
int model_gemm(Model* m, int epi, const CUtensorMap& map, const void* w, const void* x, int n_tok, int n_out, int k,
               int up_offset, const void* res, void* y, cudaStream_t s) {
  const EesdModelDesc& d = m->d;
  if (d.dtype == EESD_BF16) {
    const int rc = tc_gemm_launch(epi, map, x, n_tok, n_out, k, up_offset, res, n_out, y, n_out, m->keys,
                                  m->status, s, d.weights_packed, m->gemm_scratch);
    m->launches += 1;
    return rc ? fail(rc, "tcgen05 gemm launch failed (n_tok=%d n_out=%d k=%d epi=%d)", n_tok, n_out, k, epi) : 0;
  }
  if (epi == EESD_EPI_SWIGLU) {
    int rc = launch_simt_gemm_f32(EESD_EPI_STORE, (const float*)x, (const float*)w, nullptr, m->gu, n_tok,
                                  2 * d.intermediate, k, s);
    if (!rc) rc = launch_swiglu_f32(m->gu, (float*)y, n_tok, d.intermediate, s);
    m->launches += 2;
    return rc ? fail(rc, "fp32 gemm+swiglu launch failed") : 0;
  }
  const int rc = launch_simt_gemm_f32(epi, (const float*)x, (const float*)w, (const float*)res, (float*)y, n_tok, n_out,
                                      k, s);
  m->launches += 1;
  return rc ? fail(rc, "fp32 gemm launch failed") : 0;
}

int check_batch(const Model* m, const EesdBatch* b) {
  if (!b || b->n_tokens < 0 || b->n_tokens > m->d.max_tokens)
    return fail(EESD_ERR_ARG, "batch: n_tokens %d outside [0, %d]", b ? b->n_tokens : -1, m->d.max_tokens);
  if (b->n_tokens && (!b->tok_pos || !b->tok_row || !b->blk || !b->items || b->n_blocks <= 0 || b->n_items <= 0))
    return fail(EESD_ERR_ARG, "batch: missing metadata");
  if (b->max_ctx > m->d.max_seq) return fail(EESD_ERR_ARG, "batch: max_ctx %d > max_seq %d", b->max_ctx, m->d.max_seq);
  return EESD_OK;
}

}  // namespace

void set_last_error(const char* msg) { g_err = msg; }
uint32_t spin_limit() { return g_spin_limit; }

}  // namespace eesd

using namespace eesd;

extern "C" {

int eesd_version(void) { return EESD_VERSION; }
const char* eesd_last_error(void) { return g_err.c_str(); }

int eesd_attn_item_tokens(int n_heads, int n_kv_heads) {
  if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads) return -1;
  return attn_item_tokens(n_heads, n_kv_heads);
}

size_t eesd_model_workspace_bytes(const EesdModelDesc* d) { return d ? layout_for(*d).total : 0; }

int eesd_model_create(const EesdModelDesc* d, void** out) {
  if (!d || !out) return fail(EESD_ERR_ARG, "null argument");
  *out = nullptr;
  if (d->dtype != EESD_BF16 && d->dtype != EESD_F32) return fail(EESD_ERR_ARG, "dtype %d", d->dtype);
  if (d->n_layers <= 0 || d->dim <= 0 || d->n_heads <= 0 || d->n_kv_heads <= 0 || d->n_heads % d->n_kv_heads ||
      (d->head_dim != 64 && d->head_dim != 128) || d->intermediate <= 0 || d->vocab <= 0)
    return fail(EESD_ERR_ARG, "unsupported model shape (head_dim must be 64 or 128)");
  if (d->max_seq % 64 || d->max_batch <= 0 || d->max_tokens <= 0) return fail(EESD_ERR_ARG, "bad cache/batch sizes");
  if (d->dtype == EESD_BF16 && (d->dim % 64 || d->intermediate % 64 || (d->n_heads * d->head_dim) % 64))
    return fail(EESD_ERR_ARG, "bf16 path needs dim, intermediate and Hq*D multiples of 64");
  if (d->weights_packed && (d->dtype != EESD_BF16 || d->intermediate % 128))
    return fail(EESD_ERR_ARG, "packed weights need bf16 and intermediate %% 128 == 0");
  const Layout L = layout_for(*d);
  if (!d->workspace || d->workspace_bytes < L.total)
    return fail(EESD_ERR_ARG, "workspace too small: %zu < %zu", d->workspace_bytes, L.total);
  if (reinterpret_cast<uintptr_t>(d->workspace) & 255) return fail(EESD_ERR_ARG, "workspace not 256-byte aligned");
  Model* m = new Model();
  m->d = *d;
  m->eb = d->dtype == EESD_BF16 ? 2 : 4;
  m->q_dim = d->n_heads * d->head_dim;
  m->qkv_dim = (d->n_heads + 2 * d->n_kv_heads) * d->head_dim;
  for (int i = 0; i < d->n_layers; ++i) {
    m->wqkv.push_back(d->wqkv[i]);
    m->wo.push_back(d->wo[i]);
    m->w13.push_back(d->w13[i]);
    m->w2.push_back(d->w2[i]);
    m->attn_norm.push_back(d->attn_norm[i]);
    m->ffn_norm.push_back(d->ffn_norm[i]);
  }
  // the descriptor's pointer arrays belong to the caller: keep our own copies only
  m->d.wqkv = m->d.wo = m->d.w13 = m->d.w2 = m->d.attn_norm = m->d.ffn_norm = nullptr;
  uint8_t* ws = static_cast<uint8_t*>(d->workspace);
  m->status = reinterpret_cast<int*>(ws + L.status);
  m->xn = ws + L.xn;
  m->qkv = ws + L.qkv;
  m->attn = ws + L.attn;
  m->act = ws + L.act;
  m->gu = reinterpret_cast<float*>(ws + L.gu);
  m->logits32 = reinterpret_cast<float*>(ws + L.logits32);
  m->keys = reinterpret_cast<unsigned long long*>(ws + L.keys);
  m->attn_order = reinterpret_cast<int32_t*>(ws + L.order);
  m->gemm_scratch.partials = ws + L.partials;
  m->gemm_scratch.partial_bytes = L.partial_bytes;
  if (d->dtype == EESD_BF16) {
    m->map_qkv.resize(d->n_layers);
    m->map_o.resize(d->n_layers);
    m->map_13.resize(d->n_layers);
    m->map_2.resize(d->n_layers);
    auto enc = [&](CUtensorMap* map, const void* w, int rows, int k) {
      return d->weights_packed ? encode_packed_map(map, w, rows, k) : encode_kmajor_map(map, w, rows, k, 128);
    };
    for (int i = 0; i < d->n_layers; ++i) {
      int rc = enc(&m->map_qkv[i], m->wqkv[i], m->qkv_dim, d->dim);
      if (!rc) rc = enc(&m->map_o[i], m->wo[i], d->dim, m->q_dim);
      if (!rc) rc = enc(&m->map_13[i], m->w13[i], 2 * d->intermediate, d->dim);
      if (!rc) rc = enc(&m->map_2[i], m->w2[i], d->dim, d->intermediate);
      if (rc) {
        delete m;
        return fail(rc, "tensor map encode failed for layer %d (16-byte aligned weights required)", i);
      }
    }
    if (enc(&m->map_head, d->lm_head, d->vocab, d->dim)) {
      delete m;
      return fail(EESD_ERR_CUDA, "tensor map encode failed for the LM head");
    }
    const long long cache_rows = (long long)d->n_layers * d->max_batch * d->n_kv_heads * d->max_seq;
    if (cache_rows >= (1LL << 31)) {
      delete m;
      return fail(EESD_ERR_ARG, "KV cache too large for 32-bit TMA row coordinates");
    }
    if (encode_kmajor_map(&m->map_kc, d->k_cache, (int)cache_rows, d->head_dim, 64) ||
        encode_kmajor_map(&m->map_vc, d->v_cache, (int)cache_rows, d->head_dim, 64)) {
      delete m;
      return fail(EESD_ERR_CUDA, "tensor map encode failed for the KV cache");
    }
  }
  // the status word starts at zero
  cudaError_t e = cudaMemset(ws + L.status, 0, 256);
  if (e != cudaSuccess) {
    delete m;
    return cuda_fail(e, "workspace init");
  }
  *out = m;
  return EESD_OK;
}

int eesd_model_destroy(void* h) {
  Model* m = static_cast<Model*>(h);
  if (!m) return EESD_OK;
  for (cudaEvent_t e : m->pool) cudaEventDestroy(e);
  delete m;
  return EESD_OK;
}

int eesd_forward_layers(void* h, void* x, const EesdBatch* b, int start, int end, void* stream) {
  Model* m = static_cast<Model*>(h);
  if (!m || !x) return fail(EESD_ERR_ARG, "null model or x");
  int rc = check_batch(m, b);
  if (rc) return rc;
  const EesdModelDesc& d = m->d;
  if (start < 0 || end > d.n_layers || start > end) return fail(EESD_ERR_ARG, "layer range [%d, %d)", start, end);
  const int N = b->n_tokens;
  if (N == 0 || start == end) return EESD_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t layer_kv = (size_t)d.max_batch * d.n_kv_heads * d.max_seq * d.head_dim * m->eb;
  AttnGeom g{d.n_heads, d.n_kv_heads, d.head_dim, d.max_batch, d.max_seq, m->qkv_dim,
             1.0f / sqrtf((float)d.head_dim), N, b->n_blocks, 0u, nullptr};
  ProfEvent pe;
  // query rows of the largest attention work item: one token per block (draft) or up to a full item
  const int G = d.n_heads / d.n_kv_heads;
  const int rows_max = b->n_tokens == b->n_blocks ? G : attn_item_tokens(d.n_heads, d.n_kv_heads) * G;
  if (d.dtype == EESD_BF16 && b->n_items <= kAttnOrderMax) {
    // every layer's attention grid runs the batch's work items longest first
    rc = launch_attn_order(b->blk, b->items, b->n_items, b->n_blocks, d.n_heads, d.n_kv_heads, m->attn_order, s);
    m->launches++;
    if (rc) return fail(rc, "attention order launch");
    g.order = m->attn_order;
  }
  for (int i = start; i < end; ++i) {
    uint8_t* kc = static_cast<uint8_t*>(d.k_cache) + (size_t)i * layer_kv;
    uint8_t* vc = static_cast<uint8_t*>(d.v_cache) + (size_t)i * layer_kv;
    prof_begin(m, s, EESD_PROF_NORM, &pe, N);
    rc = launch_rmsnorm(d.dtype, x, nullptr, m->attn_norm[i], m->xn, N, d.dim, d.norm_eps, s);
    prof_end(m, s, &pe);
    m->launches++;
    if (rc) return fail(rc, "rmsnorm launch");
    prof_begin(m, s, EESD_PROF_GEMM_QKV, &pe, N);
    rc = model_gemm(m, EESD_EPI_STORE, m->map_qkv.empty() ? m->map_head : m->map_qkv[i], m->wqkv[i], m->xn, N,
                    m->qkv_dim, d.dim, 0, nullptr, m->qkv, s);
    prof_end(m, s, &pe);
    if (rc) return rc;
    // Draft and verify batches (every block one attention work item): the attention kernel does
    // RoPE and the KV append itself.  Batches with longer blocks (prefill) use the RoPE/KV kernel.
    AttnAppend app;
    app.on = d.dtype == EESD_BF16 && b->n_items == b->n_blocks;
    if (app.on) {
      app.kc = kc;
      app.vc = vc;
      app.cos = d.rope_cos;
      app.sin = d.rope_sin;
    } else {
      prof_begin(m, s, EESD_PROF_ROPE_KV, &pe, N);
      rc = launch_rope_kv(d.dtype, m->qkv, b->tok_pos, b->tok_row, N, d.n_heads, d.n_kv_heads, d.head_dim, d.rope_cos,
                          d.rope_sin, kc, vc, d.max_batch, d.max_seq, m->status, s);
      prof_end(m, s, &pe);
      m->launches++;
      if (rc) return fail(rc, "rope/kv launch");
    }
    prof_begin(m, s, EESD_PROF_ATTN, &pe, N);
    rc = launch_attention(d.dtype, g, m->qkv, d.k_cache, d.v_cache, m->attn, b->blk, b->items, b->n_items, b->max_ctx,
                          m->status, s, &m->map_kc, &m->map_vc, i, app, rows_max);
    prof_end(m, s, &pe);
    m->launches++;
    if (rc) return fail(rc, "attention launch");
    prof_begin(m, s, EESD_PROF_GEMM_O, &pe, N);
    rc = model_gemm(m, EESD_EPI_RESIDUAL, m->map_o.empty() ? m->map_head : m->map_o[i], m->wo[i], m->attn, N, d.dim,
                    m->q_dim, 0, x, x, s);
    prof_end(m, s, &pe);
    if (rc) return rc;
    prof_begin(m, s, EESD_PROF_NORM, &pe, N);
    rc = launch_rmsnorm(d.dtype, x, nullptr, m->ffn_norm[i], m->xn, N, d.dim, d.norm_eps, s);
    prof_end(m, s, &pe);
    m->launches++;
    if (rc) return fail(rc, "rmsnorm launch");
    prof_begin(m, s, EESD_PROF_GEMM_W13, &pe, N);
    rc = model_gemm(m, EESD_EPI_SWIGLU, m->map_13.empty() ? m->map_head : m->map_13[i], m->w13[i], m->xn, N,
                    d.intermediate, d.dim, d.intermediate, nullptr, m->act, s);
    prof_end(m, s, &pe);
    if (rc) return rc;
    prof_begin(m, s, EESD_PROF_GEMM_W2, &pe, N);
    rc = model_gemm(m, EESD_EPI_RESIDUAL, m->map_2.empty() ? m->map_head : m->map_2[i], m->w2[i], m->act, N, d.dim,
                    d.intermediate, 0, x, x, s);
    prof_end(m, s, &pe);
    if (rc) return rc;
  }
  return EESD_OK;
}

int eesd_head_argmax(void* h, const void* x, const int32_t* rows, int n, int32_t* out_ids, void* logits, void* stream) {
  Model* m = static_cast<Model*>(h);
  if (!m || !x || !out_ids) return fail(EESD_ERR_ARG, "null argument");
  const EesdModelDesc& d = m->d;
  if (n < 0 || n > d.max_tokens) return fail(EESD_ERR_ARG, "head rows %d outside [0, %d]", n, d.max_tokens);
  if (n == 0) return EESD_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProfEvent pe;
  prof_begin(m, s, EESD_PROF_HEAD, &pe, n);
  int rc = launch_rmsnorm(d.dtype, x, rows, d.final_norm, m->xn, n, d.dim, d.norm_eps, s);
  m->launches++;
  if (rc) return fail(rc, "head rmsnorm launch");
  if (d.dtype == EESD_BF16) {
    if (logits) {
      rc = model_gemm(m, EESD_EPI_STORE, m->map_head, d.lm_head, m->xn, n, d.vocab, d.dim, 0, nullptr, logits, s);
      if (!rc) rc = launch_argmax_rows(d.dtype, logits, n, d.vocab, out_ids, s);
      m->launches++;
    } else {
      cudaError_t e = cudaMemsetAsync(m->keys, 0, (size_t)n * 8, s);
      if (e != cudaSuccess) return cuda_fail(e, "argmax key reset");
      rc = model_gemm(m, EESD_EPI_ARGMAX_INTERNAL, m->map_head, d.lm_head, m->xn, n, d.vocab, d.dim, 0, nullptr,
                      nullptr, s);
      if (!rc) rc = launch_keys_to_ids(m->keys, out_ids, n, s);
      m->launches++;
    }
  } else {
    for (int r0 = 0; r0 < n && !rc; r0 += kHeadChunk) {
      const int c = std::min(kHeadChunk, n - r0);
      float* lg = logits ? static_cast<float*>(logits) + (size_t)r0 * d.vocab : m->logits32;
      rc = launch_simt_gemm_f32(EESD_EPI_STORE, static_cast<const float*>(m->xn) + (size_t)r0 * d.dim,
                                static_cast<const float*>(d.lm_head), nullptr, lg, c, d.vocab, d.dim, s);
      if (!rc) rc = launch_argmax_rows(d.dtype, lg, c, d.vocab, out_ids + r0, s);
      m->launches += 2;
    }
  }
  prof_end(m, s, &pe);
  return rc ? fail(rc, "head launch failed") : EESD_OK;
}

int eesd_embed(void* h, const int32_t* ids, int n, void* x, void* stream) {
  Model* m = static_cast<Model*>(h);
  if (!m || !ids || !x) return fail(EESD_ERR_ARG, "null argument");
  if (n < 0) return fail(EESD_ERR_ARG, "n < 0");
  m->launches++;
  const int rc = launch_embed(m->d.dtype, m->d.embed, ids, n, m->d.dim, m->d.vocab, x, m->status,
                              static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, "embed launch") : EESD_OK;
}

int eesd_model_check(void* h, int* bits_out, void* stream) {
  Model* m = static_cast<Model*>(h);
  if (!m) return fail(EESD_ERR_ARG, "null model");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int bits = 0;
  cudaError_t e = cudaMemcpyAsync(&bits, m->status, 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && bits) e = cudaMemsetAsync(m->status, 0, 4, s);
  if (e != cudaSuccess) return cuda_fail(e, "status read");
  if (bits_out) *bits_out = bits;
  return bits ? fail(EESD_ERR_DEVICE, "device status bits 0x%x", bits) : EESD_OK;
}

int eesd_model_profile(void* h, int enable) {
  Model* m = static_cast<Model*>(h);
  if (!m) return fail(EESD_ERR_ARG, "null model");
  m->prof = enable != 0;
  m->events.clear();
  m->pool_used = 0;
  return EESD_OK;
}

int eesd_model_profile_read(void* h, double* ms, int64_t* launches) {
  Model* m = static_cast<Model*>(h);
  if (!m || !ms || !launches) return fail(EESD_ERR_ARG, "null argument");
  for (int k = 0; k < EESD_PROF_KINDS; ++k) {
    ms[k] = 0;
    launches[k] = 0;
  }
  for (const ProfEvent& e : m->events) {
    float t = 0.f;
    cudaError_t err = cudaEventSynchronize(e.b);
    if (err == cudaSuccess) err = cudaEventElapsedTime(&t, e.a, e.b);
    if (err != cudaSuccess) return cuda_fail(err, "profile event");
    ms[e.kind] += t;
    launches[e.kind] += 1;
  }
  return EESD_OK;
}

int eesd_model_profile_records(void* h, int32_t* kinds, int32_t* n_tok, float* ms, int cap) {
  Model* m = static_cast<Model*>(h);
  if (!m) return -1;
  int n = 0;
  for (const ProfEvent& e : m->events) {
    if (n >= cap) break;
    float t = 0.f;
    if (cudaEventSynchronize(e.b) != cudaSuccess || cudaEventElapsedTime(&t, e.a, e.b) != cudaSuccess) return -1;
    if (kinds) kinds[n] = e.kind;
    if (n_tok) n_tok[n] = e.n_tok;
    if (ms) ms[n] = t;
    ++n;
  }
  return n;
}

int64_t eesd_model_launch_count(void* h) {
  const Model* m = static_cast<const Model*>(h);
  return m ? m->launches : -1;
}

int eesd_copy_rows(int dtype, const void* src, const int32_t* src_idx, void* dst, const int32_t* dst_idx, int n,
                   int width, void* stream) {
  if (!src || !dst || n < 0 || width <= 0) return fail(EESD_ERR_ARG, "copy_rows arguments");
  const int rc = launch_copy_rows(dtype, src, src_idx, dst, dst_idx, n, width, static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, "copy_rows launch") : EESD_OK;
}

int eesd_gather_ids(const int32_t* table, const int32_t* idx, int32_t* ids, int n, void* stream) {
  if (!table || !idx || !ids || n < 0) return fail(EESD_ERR_ARG, "gather_ids arguments");
  const int rc = launch_gather_ids(table, idx, ids, n, static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, "gather_ids launch") : EESD_OK;
}

int eesd_scatter_ids(const int32_t* ids, const int32_t* idx, int32_t* table, int n, void* stream) {
  if (!table || !idx || !ids || n < 0) return fail(EESD_ERR_ARG, "scatter_ids arguments");
  const int rc = launch_scatter_ids(ids, idx, table, n, static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, "scatter_ids launch") : EESD_OK;
}

int eesd_greedy_accept(const int32_t* y, const int32_t* vinfo, int nv, int32_t* seq_buf, int stride, int32_t* acc,
                       void* stream) {
  if (!y || !vinfo || !seq_buf || !acc || nv < 0 || stride <= 0) return fail(EESD_ERR_ARG, "greedy_accept arguments");
  const int rc = launch_greedy_accept(y, vinfo, nv, seq_buf, stride, acc, static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, "greedy_accept launch") : EESD_OK;
}

size_t eesd_round_meta_ints(int n, int gamma, int item_tokens) {
  if (n < 0 || gamma < 0 || item_tokens <= 0) return 0;
  const size_t cols = (size_t)gamma + 1, ni = (cols + item_tokens - 1) / item_tokens;
  return cols * 10 * (size_t)n + (size_t)n * (3 * cols + 4 + 2 * ni + 3);
}

int eesd_round_meta(const int32_t* act, int n, const int32_t* pos, int max_batch, int gamma, int item_tokens,
                    int32_t* out, void* stream) {
  if (!act || !pos || !out || n < 0 || max_batch <= 0 || gamma < 0 || item_tokens <= 0)
    return fail(EESD_ERR_ARG, "round_meta arguments");
  const int rc = launch_round_meta(act, n, pos, max_batch, gamma + 1, item_tokens, out, static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, "round_meta launch") : EESD_OK;
}

int eesd_round_advance(const int32_t* act, int n, const int32_t* acc, int32_t* pos, int max_batch, void* stream) {
  if (!act || !acc || !pos || n < 0 || max_batch <= 0) return fail(EESD_ERR_ARG, "round_advance arguments");
  const int rc = launch_round_advance(act, n, acc, pos, max_batch, static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, "round_advance launch") : EESD_OK;
}

int eesd_rmsnorm(int dtype, const void* x, const int32_t* rows, const void* w, void* y, int n, int dim, float eps,
                 void* stream) {
  if (!x || !w || !y || n < 0 || dim <= 0) return fail(EESD_ERR_ARG, "rmsnorm arguments");
  const int rc = launch_rmsnorm(dtype, x, rows, w, y, n, dim, eps, static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, "rmsnorm launch") : EESD_OK;
}

size_t eesd_gemm_workspace_bytes(int n_tok, int n_out, int k, int epilogue) {
  if (n_tok <= 0 || n_out <= 0 || k <= 0) return 0;
  size_t b = 256;                                                                  // status word
  if (epilogue == EESD_EPI_SWIGLU) b += align256((size_t)n_tok * 2 * n_out * 4);   // fp32 path scratch
  if (k % 64 == 0) b += align256(tc_plan(n_tok, n_out, k, epilogue).partial_bytes);  // bf16 split-K scratch
  return b;
}

int eesd_gemm(int dtype, int epilogue, const void* x, const void* w, const void* residual, void* y, int n_tok,
              int n_out, int k, int up_offset, void* workspace, size_t workspace_bytes, void* stream) {
  if (!x || !w || !y || n_tok <= 0 || n_out <= 0 || k <= 0) return fail(EESD_ERR_ARG, "gemm arguments");
  if (epilogue < EESD_EPI_STORE || epilogue > EESD_EPI_SWIGLU) return fail(EESD_ERR_ARG, "epilogue %d", epilogue);
  if (epilogue == EESD_EPI_RESIDUAL && !residual) return fail(EESD_ERR_ARG, "residual epilogue needs residual");
  const size_t need = eesd_gemm_workspace_bytes(n_tok, n_out, k, epilogue);
  if (!workspace || workspace_bytes < need) return fail(EESD_ERR_ARG, "gemm workspace %zu < %zu", workspace_bytes, need);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* status = reinterpret_cast<int*>(ws);
  if (dtype != EESD_BF16 && dtype != EESD_F32) return fail(EESD_ERR_ARG, "dtype %d", dtype);
  cudaError_t e = cudaMemsetAsync(ws, 0, 256, s);
  if (e != cudaSuccess) return cuda_fail(e, "gemm status reset");
  if (dtype == EESD_BF16) {
    if (k % 64) return fail(EESD_ERR_ARG, "bf16 gemm needs k %% 64 == 0");
    TcScratch sc;
    sc.partials = ws + 256 + (epilogue == EESD_EPI_SWIGLU ? align256((size_t)n_tok * 2 * n_out * 4) : 0);
    sc.partial_bytes = tc_plan(n_tok, n_out, k, epilogue).partial_bytes;
    CUtensorMap map;
    const int rows = epilogue == EESD_EPI_SWIGLU ? up_offset + n_out : n_out;
    int rc = encode_kmajor_map(&map, w, rows, k, 128);
    if (rc) return fail(rc, "weight tensor map");
    rc = tc_gemm_launch(epilogue, map, x, n_tok, n_out, k, up_offset, residual, n_out, y, n_out, nullptr, status, s, 0,
                        sc);
    return rc ? fail(rc, "tcgen05 gemm launch") : EESD_OK;
  }
  int rc;
  if (epilogue == EESD_EPI_SWIGLU) {
    float* gu = reinterpret_cast<float*>(ws + 256);
    if (up_offset != n_out) return fail(EESD_ERR_ARG, "fp32 swiglu needs up_offset == n_out");
    rc = launch_simt_gemm_f32(EESD_EPI_STORE, (const float*)x, (const float*)w, nullptr, gu, n_tok, 2 * n_out, k, s);
    if (!rc) rc = launch_swiglu_f32(gu, (float*)y, n_tok, n_out, s);
  } else {
    rc = launch_simt_gemm_f32(epilogue, (const float*)x, (const float*)w, (const float*)residual, (float*)y, n_tok,
                              n_out, k, s);
  }
  return rc ? fail(rc, "fp32 gemm launch") : EESD_OK;
}

size_t eesd_packed_weight_bytes(int rows, int k) {
  return (rows > 0 && k > 0 && k % 64 == 0) ? packed_weight_bytes(rows, k) : 0;
}

int eesd_pack_weight(const void* w, int rows, int k, void* out, void* stream) {
  const int rc = pack_weight(w, rows, k, out, static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, "pack_weight: rows %d k %d (k %% 64 == 0, 16-byte aligned pointers)", rows, k) : EESD_OK;
}

int eesd_status_read(const int32_t* status, int* bits_out, void* stream) {
  if (!status) return fail(EESD_ERR_ARG, "null status");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int bits = 0;
  cudaError_t e = cudaMemcpyAsync(&bits, status, 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "status read");
  if (bits_out) *bits_out = bits;
  return bits ? fail(EESD_ERR_DEVICE, "device status bits 0x%x", bits) : EESD_OK;
}

int eesd_attn_varlen_gqa(int dtype, const void* qkv, int n_heads, int n_kv_heads, int head_dim, void* k_cache,
                         void* v_cache, int max_batch, int max_seq, const EesdBatch* b, int append,
                         const float* rope_cos, const float* rope_sin, void* out, int32_t* status, void* stream) {
  if (!qkv || !k_cache || !v_cache || !out || !b) return fail(EESD_ERR_ARG, "attn: null argument");
  if (dtype != EESD_BF16 && dtype != EESD_F32) return fail(EESD_ERR_ARG, "attn: dtype %d", dtype);
  if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || (head_dim != 64 && head_dim != 128))
    return fail(EESD_ERR_ARG, "attn: heads %d / %d, head_dim %d (64 or 128)", n_heads, n_kv_heads, head_dim);
  if (max_batch <= 0 || max_seq <= 0 || max_seq % 64) return fail(EESD_ERR_ARG, "attn: max_seq must be a multiple of 64");
  if (b->n_tokens < 0 || b->n_blocks < 0 || b->n_items < 0) return fail(EESD_ERR_ARG, "attn: negative batch sizes");
  if (b->n_tokens == 0 || b->n_items == 0) return EESD_OK;
  if (!b->blk || !b->items || b->n_blocks <= 0) return fail(EESD_ERR_ARG, "attn: missing block metadata");
  if (b->max_ctx > max_seq) return fail(EESD_ERR_ARG, "attn: max_ctx %d > max_seq %d", b->max_ctx, max_seq);
  const long long cache_rows = (long long)max_batch * n_kv_heads * max_seq;
  if (cache_rows >= (1LL << 31)) return fail(EESD_ERR_ARG, "attn: cache too large for 32-bit TMA row coordinates");
  AttnAppend app;
  if (append) {
    if (dtype != EESD_BF16) return fail(EESD_ERR_ARG, "attn: the in-kernel RoPE/append path is bf16 only");
    if (b->n_items != b->n_blocks)
      return fail(EESD_ERR_ARG, "attn: append needs every block to be one work item (n_items == n_blocks)");
    if (!rope_cos || !rope_sin) return fail(EESD_ERR_ARG, "attn: append needs the RoPE tables");
    app.on = true;
    app.kc = k_cache;
    app.vc = v_cache;
    app.cos = rope_cos;
    app.sin = rope_sin;
  }
  const int qkv_dim = (n_heads + 2 * n_kv_heads) * head_dim;
  AttnGeom g{n_heads, n_kv_heads, head_dim, max_batch, max_seq, qkv_dim, 1.0f / sqrtf((float)head_dim), b->n_tokens,
             b->n_blocks, 0u, nullptr};
  CUtensorMap kmap, vmap;
  if (dtype == EESD_BF16) {
    if (encode_kmajor_map(&kmap, k_cache, (int)cache_rows, head_dim, 64) ||
        encode_kmajor_map(&vmap, v_cache, (int)cache_rows, head_dim, 64))
      return fail(EESD_ERR_ARG, "attn: KV cache tensor map (16-byte aligned bf16 caches required)");
  }
  const int G = n_heads / n_kv_heads;
  const int rows_max = b->n_tokens == b->n_blocks ? G : attn_item_tokens(n_heads, n_kv_heads) * G;
  const int rc = launch_attention(dtype, g, qkv, k_cache, v_cache, out, b->blk, b->items, b->n_items, b->max_ctx,
                                  status, static_cast<cudaStream_t>(stream), &kmap, &vmap, 0, app, rows_max);
  return rc ? fail(rc, "attention launch") : EESD_OK;
}

int eesd_rope_kv_append(int dtype, void* qkv, const int32_t* tok_pos, const int32_t* tok_row, int n_tok, int n_heads,
                        int n_kv_heads, int head_dim, const float* rope_cos, const float* rope_sin, void* k_cache,
                        void* v_cache, int max_batch, int max_seq, int32_t* status, void* stream) {
  if (!qkv || !tok_pos || !tok_row || !rope_cos || !rope_sin || !k_cache || !v_cache || n_tok < 0)
    return fail(EESD_ERR_ARG, "rope_kv_append: null argument or n_tok < 0");
  if (dtype != EESD_BF16 && dtype != EESD_F32) return fail(EESD_ERR_ARG, "rope_kv_append: dtype %d", dtype);
  if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || (head_dim != 64 && head_dim != 128))
    return fail(EESD_ERR_ARG, "rope_kv_append: heads %d / %d, head_dim %d", n_heads, n_kv_heads, head_dim);
  if (max_batch <= 0 || max_seq <= 0) return fail(EESD_ERR_ARG, "rope_kv_append: cache sizes");
  const int rc = launch_rope_kv(dtype, qkv, tok_pos, tok_row, n_tok, n_heads, n_kv_heads, head_dim, rope_cos, rope_sin,
                                k_cache, v_cache, max_batch, max_seq, status, static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, "rope_kv_append launch") : EESD_OK;
}

int eesd_set_option(int option, int value) {
  if (option == 1) {   // tcgen05 MMA N: 0 = whole token tile, else a fixed multiple of 16
    if (value < 0 || value > 256 || value % 16) return fail(EESD_ERR_ARG, "mma n %d", value);
    tc_set_mma_n(value);
    return EESD_OK;
  }
  if (option == 2) {   // tcgen05 split-K count: 0 = from the weight shape (changes summation order)
    if (value < 0 || value > 8) return fail(EESD_ERR_ARG, "splits %d", value);
    tc_set_splits(value);
    return EESD_OK;
  }
  if (option == 3) {   // tcgen05 pipeline stages: 0 = as many as fit
    if (value < 0 || value > 8 || value == 1) return fail(EESD_ERR_ARG, "stages %d", value);
    tc_set_stages(value);
    return EESD_OK;
  }
  if (option == 4) {   // tcgen05 CTA pairs for SwiGLU GEMMs: 1 = on (default), 0 = off (numerics-neutral)
    if (value < 0 || value > 1) return fail(EESD_ERR_ARG, "pair %d", value);
    tc_set_pair(value);
    return EESD_OK;
  }
  if (option == 5) {   // LM head: two row tiles per CTA up to 256 tokens: 1 = on (default), 0 = off
    if (value < 0 || value > 1) return fail(EESD_ERR_ARG, "head two tiles %d", value);
    tc_set_head_two_tiles(value);
    return EESD_OK;
  }
  if (option == 7) {   // N of the first of two MMAs per k-step for token tiles above 256 (default 192; 0: halves)
    if (value < 0 || value > 256 || value % 16) return fail(EESD_ERR_ARG, "split n %d", value);
    tc_set_split_n(value);
    return EESD_OK;
  }
  if (option == 6) {   // pipeline-wait poll limit: -1 = the default, n >= 0 = n polls (0: every wait gives up)
    if (value < -1) return fail(EESD_ERR_ARG, "spin limit %d", value);
    g_spin_limit = value < 0 ? kSpinLimit : (uint32_t)value;
    return EESD_OK;
  }
  return fail(EESD_ERR_ARG, "unknown option %d", option);
}

}  // extern "C"
