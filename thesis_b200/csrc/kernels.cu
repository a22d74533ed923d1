// Non-GEMM kernels of the packed draft/verify step: RMSNorm, RoPE + in-place KV append,
// varlen GQA attention over the static per-row KV cache, embedding / row gathers, greedy
// acceptance, argmax, and the fp32 (CUDA-core) GEMM of the parity path.
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace eesd {

namespace {

// 2^x with the hardware approximation (ex2.approx; 2^-inf = 0)
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------- RMSNorm (common/model.py:153-156)
// y = w * round(x * rsqrt(mean(x^2) + eps)); the sum of squares has a fixed per-row order
// (fixed per-thread chunks, then a fixed tree), so a row's result never depends on which other
// rows share the launch.  bf16 rows of dim <= 8 * 256 * kVec are held in registers between the
// two passes (16-byte loads).
// With a row list, a source row outside [0, n_src) sets kStatusBadIndex and its output row is zeroed.
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const T* __restrict__ x, const int32_t* __restrict__ rows,
                                                      const T* __restrict__ w, T* __restrict__ y, int dim, float eps,
                                                      int n_src, int* status) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[8];
  const int i = blockIdx.x;
  const int src = rows ? rows[i] : i;
  if (src < 0 || src >= n_src) {
    if (threadIdx.x == 0) set_status(status, kStatusBadIndex);
    for (int j = threadIdx.x; j < dim; j += 256) y[(size_t)i * dim + j] = from_f<T>(0.f);
    return;
  }
  const T* xr = x + (size_t)src * dim;
  T* yr = y + (size_t)i * dim;
  constexpr int EPV = 16 / sizeof(T);              // elements per 16-byte vector
  constexpr int kVec = 4;                           // vectors per thread held in registers
  const bool vec = (dim % EPV) == 0 && dim <= 256 * EPV * kVec &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y)) &
                    15) == 0;
  float ss = 0.f;
  uint4 buf[kVec];
  if (vec) {
    const int nv = dim / EPV;
#pragma unroll
    for (int k = 0; k < kVec; ++k) {
      const int vi = threadIdx.x + k * 256;
      if (vi < nv) {
        buf[k] = reinterpret_cast<const uint4*>(xr)[vi];
        const T* e = reinterpret_cast<const T*>(&buf[k]);
#pragma unroll
        for (int j = 0; j < EPV; ++j) {
          const float v = to_f(e[j]);
          ss = fmaf(v, v, ss);
        }
      }
    }
  } else {
    for (int j = threadIdx.x; j < dim; j += 256) {
      const float v = to_f(xr[j]);
      ss = fmaf(v, v, ss);
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int k = 0; k < 8; ++k) t += red[k];
    red[0] = rsqrtf(t / (float)dim + eps);
  }
  __syncthreads();
  const float r = red[0];
  if (vec) {
    const int nv = dim / EPV;
#pragma unroll
    for (int k = 0; k < kVec; ++k) {
      const int vi = threadIdx.x + k * 256;
      if (vi < nv) {
        const uint4 wv = reinterpret_cast<const uint4*>(w)[vi];
        const T* e = reinterpret_cast<const T*>(&buf[k]);
        const T* we = reinterpret_cast<const T*>(&wv);
        uint4 ov;
        T* oe = reinterpret_cast<T*>(&ov);
#pragma unroll
        for (int j = 0; j < EPV; ++j) oe[j] = from_f<T>(to_f(we[j]) * rnd<T>(to_f(e[j]) * r));
        reinterpret_cast<uint4*>(yr)[vi] = ov;
      }
    }
  } else {
    for (int j = threadIdx.x; j < dim; j += 256) yr[j] = from_f<T>(to_f(w[j]) * rnd<T>(to_f(xr[j]) * r));
  }
}

// ---------------------------------------------------------------- RoPE + KV append
// common/model.py:143-150 and solutions/packed.py:176-181: q, k rotated in the rotate-half
// layout with cos/sin cast to the model dtype; q written back in place, k and v written into
// the cache at (row, kv head, position).  Rollback needs no kernel: stale positions beyond a
// row's committed length are never read.  One CTA per token; thread t owns rotation pair
// d = t % (D/2) of heads t / (D/2), t / (D/2) + 256 / (D/2), ... so the table entries are read once.
template <typename T>
__global__ void __launch_bounds__(256) rope_kv_kernel(T* __restrict__ qkv, const int32_t* __restrict__ tok_pos,
                                                      const int32_t* __restrict__ tok_row, int n_heads,
                                                      int n_kv_heads, int D, const float* __restrict__ cosb,
                                                      const float* __restrict__ sinb, T* __restrict__ kc,
                                                      T* __restrict__ vc, int max_batch, int max_seq, int* status) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int pos = tok_pos[t], row = tok_row[t];
  if (pos < 0 || pos >= max_seq || row < 0 || row >= max_batch) {
    if (threadIdx.x == 0) set_status(status, kStatusBadIndex);
    return;
  }
  const int half = D / 2;
  const int ldq = (n_heads + 2 * n_kv_heads) * D;
  T* base = qkv + (size_t)t * ldq;
  const int d = threadIdx.x % half;
  const int h0 = threadIdx.x / half, hstep = blockDim.x / half;
  const float c1 = rnd<T>(cosb[(size_t)pos * D + d]), c2 = rnd<T>(cosb[(size_t)pos * D + d + half]);
  const float s1 = rnd<T>(sinb[(size_t)pos * D + d]), s2 = rnd<T>(sinb[(size_t)pos * D + d + half]);
  for (int h = h0; h < n_heads + n_kv_heads; h += hstep) {
    T* xh = base + h * D;     // heads 0..Hq-1 are q, Hq.. are k (contiguous in the fused row)
    const float x1 = to_f(xh[d]), x2 = to_f(xh[d + half]);
    const T o1 = from_f<T>(rnd<T>(x1 * c1) + rnd<T>(-x2 * s1));
    const T o2 = from_f<T>(rnd<T>(x2 * c2) + rnd<T>(x1 * s2));
    if (h < n_heads) {
      xh[d] = o1;
      xh[d + half] = o2;
    } else {
      T* dst = kc + (((size_t)row * n_kv_heads + (h - n_heads)) * max_seq + pos) * D;
      dst[d] = o1;
      dst[d + half] = o2;
    }
  }
  const T* v = base + (n_heads + n_kv_heads) * D;
  constexpr int EPV = 16 / sizeof(T);
  const int nvec = n_kv_heads * D / EPV;
  for (int idx = threadIdx.x; idx < nvec; idx += blockDim.x) {
    const int e = idx * EPV;
    const int h = e / D, dd = e - h * D;
    *reinterpret_cast<uint4*>(&vc[(((size_t)row * n_kv_heads + h) * max_seq + pos) * D + dd]) =
        reinterpret_cast<const uint4*>(v)[idx];
  }
}

// ---------------------------------------------------------------- attention
// One CTA per (work item, KV head).  A work item is up to `item_tokens` consecutive tokens of
// one block; its query rows are (token, q head of this KV group), GQA folded into rows as in
// solutions/packed.py:158.  Key tiles start at absolute position 0 and are visited in order,
// so a query's result does not depend on the other queries of the launch (a fully masked
// tile leaves the running max, sum and output unchanged).

// A work item's block must lie inside the launch's tokens and its key range inside its cache row
// (the exported attention entry point takes caller-built metadata); an invalid item sets
// kStatusBadIndex and its CTA returns before touching memory.
__device__ __forceinline__ bool attn_item_ok(const AttnGeom& g, int b, int t0, int start, int T, int row, int pos0) {
  return b >= 0 && b < g.n_blocks && T > 0 && t0 >= 0 && t0 < T && start >= 0 && start + T <= g.n_tokens &&
         row >= 0 && row < g.max_batch && pos0 >= 0 && pos0 + T <= g.max_seq;
}

// fp32 (parity path): scalar online softmax, one warp per query row.
template <int D>
__global__ void __launch_bounds__(128) attn_f32_kernel(AttnGeom g, int item_tokens, const float* __restrict__ q,
                                                       const float* __restrict__ kc, const float* __restrict__ vc,
                                                       float* __restrict__ out, const int32_t* __restrict__ blk,
                                                       const int32_t* __restrict__ items) {
  pdl_trigger();
  pdl_wait();
  constexpr int KT = 32, DP = D + 1, ND = D / 32, MAXR = 8;
  extern __shared__ float sm[];
  float* Qs = sm;                   // [32][D]
  float* Ks = Qs + 32 * D;          // [KT][DP]
  float* Vs = Ks + KT * DP;         // [KT][D]
  const int item = blockIdx.x, kvh = blockIdx.y;
  const int b = items[2 * item], t0 = items[2 * item + 1];
  if (b < 0 || b >= g.n_blocks) {
    if (threadIdx.x == 0) set_status(g.status, kStatusBadIndex);
    return;
  }
  const int start = blk[4 * b], T = blk[4 * b + 1], row = blk[4 * b + 2], pos0 = blk[4 * b + 3];
  if (!attn_item_ok(g, b, t0, start, T, row, pos0)) {
    if (threadIdx.x == 0) set_status(g.status, kStatusBadIndex);
    return;
  }
  const int G = g.n_heads / g.n_kv_heads;
  const int nt = min(item_tokens, T - t0);
  const int nrows = nt * G;
  const int kv_len = pos0 + t0 + nt;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int idx = threadIdx.x; idx < nrows * D; idx += blockDim.x) {
    const int r = idx / D, d = idx - r * D;
    Qs[idx] = q[(size_t)(start + t0 + r / G) * g.ld_q + (kvh * G + r % G) * D + d];
  }
  const float* Kb = kc + ((size_t)row * g.n_kv_heads + kvh) * g.max_seq * D;
  const float* Vb = vc + ((size_t)row * g.n_kv_heads + kvh) * g.max_seq * D;
  float m[MAXR], l[MAXR], acc[MAXR][ND];
#pragma unroll
  for (int i = 0; i < MAXR; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int e = 0; e < ND; ++e) acc[i][e] = 0.f;
  }
  for (int k0 = 0; k0 < kv_len; k0 += KT) {
    __syncthreads();
    for (int idx = threadIdx.x; idx < KT * D; idx += blockDim.x) {
      const int j = idx / D, d = idx - j * D;
      const bool in = k0 + j < kv_len;
      Ks[j * DP + d] = in ? Kb[(size_t)(k0 + j) * D + d] : 0.f;
      Vs[j * D + d] = in ? Vb[(size_t)(k0 + j) * D + d] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < MAXR; ++i) {
      const int r = warp + 4 * i;
      if (r < nrows) {
        const int qpos = pos0 + t0 + r / G;
        const int key = k0 + lane;
        const bool valid = key <= qpos;
        float s = -INFINITY;
        if (valid) {
          float dot = 0.f;
          for (int d = 0; d < D; ++d) dot = fmaf(Qs[r * D + d], Ks[lane * DP + d], dot);
          s = dot * g.scale;
        }
        const float mt = warp_max(s);
        const float mn = fmaxf(m[i], mt);
        const float corr = expf(m[i] - mn);
        const float p = valid ? expf(s - mn) : 0.f;
        l[i] = l[i] * corr + warp_sum(p);
#pragma unroll
        for (int e = 0; e < ND; ++e) {
          float a = acc[i][e] * corr;
          for (int j = 0; j < KT; ++j) a = fmaf(__shfl_sync(0xffffffffu, p, j), Vs[j * D + e * 32 + lane], a);
          acc[i][e] = a;
        }
        m[i] = mn;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < MAXR; ++i) {
    const int r = warp + 4 * i;
    if (r < nrows) {
      float* o = out + (size_t)(start + t0 + r / G) * g.n_heads * D + (kvh * G + r % G) * D;
#pragma unroll
      for (int e = 0; e < ND; ++e) o[e * 32 + lane] = acc[i][e] / l[i];
    }
  }
}

// bf16: tensor-core (mma.sync m16n8k16) flash-decoding over 64-key tiles staged in shared
// memory by cp.async (double buffered); each warp owns 16 query rows, softmax in fp32 registers.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool fill) {
  const int sz = fill ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Item rows <= 16 * WARPS / 4 (16-row groups).  K/V tiles of 64 keys arrive by TMA (one thread
// issues them into an NS-stage mbarrier ring; 128-byte swizzled 64-dim halves).  Warp w owns row
// group w / 4 and key quarter w % 4: it takes keys 16 (w % 4) .. +15 of every tile and keeps its
// own running max, sum and output for its rows; the four quarters' states are merged in quarter
// order at the end.  A row's arithmetic therefore depends only on its own query, its keys and the
// fixed key partition, never on the other rows of the launch or on WARPS (4 warps for one row
// group: draft steps; 8 for two: verify steps).
template <int D, int WARPS, int NS, int MINB>
__global__ void __launch_bounds__(WARPS * 32, MINB) attn_bf16_kernel(const __grid_constant__ CUtensorMap kmap,
                                                        const __grid_constant__ CUtensorMap vmap, AttnGeom g,
                                                        int item_tokens, int layer, const bf16* __restrict__ q,
                                                        bf16* __restrict__ out, const int32_t* __restrict__ blk,
                                                        const int32_t* __restrict__ items, int* status,
                                                        AttnAppend app) {
  pdl_trigger();
  pdl_wait();
  constexpr int KT = 64;              // keys per tile
  constexpr int NT = WARPS * 32;      // threads
  constexpr int RMAX = 16 * (WARPS / 4);   // query rows per item
  constexpr int HALVES = D / 64;      // 64-dim swizzled sub-tiles per K (or V) tile
  constexpr uint32_t SUB = KT * 128;  // bytes of one sub-tile (64 keys x 128 B)
  constexpr uint32_t STAGE = 2 * HALVES * SUB;
  constexpr int LDQ = D + 8;          // padded Q row (elements): conflict-free ldmatrix
  constexpr int ND = D / 8;           // output n-tiles
  constexpr int CPR = D / 8;          // 16-byte chunks per Q row
  extern __shared__ __align__(16) uint8_t smem8[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem8) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = sm;                                            // [NS][K halves | V halves]
  bf16* Qs = reinterpret_cast<bf16*>(sm + NS * STAGE);             // [RMAX][LDQ]
  uint64_t* full = reinterpret_cast<uint64_t*>(Qs + RMAX * LDQ);   // [NS]
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + NS);

  // grid (KV heads, items): the CTAs of one item are consecutive and items run in `order`
  const int kvh = blockIdx.x;
  const int item = g.order ? g.order[blockIdx.y] : (int)blockIdx.y;
  if (item < 0 || item >= g.n_items) {
    if (threadIdx.x == 0) set_status(status, kStatusBadIndex);
    return;
  }
  const int b = items[2 * item], t0 = items[2 * item + 1];
  if (b < 0 || b >= g.n_blocks) {
    if (threadIdx.x == 0) set_status(status, kStatusBadIndex);
    return;
  }
  const int start = blk[4 * b], T = blk[4 * b + 1], row = blk[4 * b + 2], pos0 = blk[4 * b + 3];
  if (!attn_item_ok(g, b, t0, start, T, row, pos0)) {
    if (threadIdx.x == 0) set_status(status, kStatusBadIndex);
    return;
  }
  const int G = g.n_heads / g.n_kv_heads;
  const int nt = min(item_tokens, T - t0);
  const int nrows = min(nt * G, RMAX);                  // the launcher picks RMAX >= nt * G
  const int kv_len = pos0 + t0 + nt;
  const int n_tiles = (kv_len + KT - 1) / KT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // first cache row of this (layer, row, kv head) in the 2-D [layers*B*Hkv*S, D] view
  const int crow = ((layer * g.max_batch + row) * g.n_kv_heads + kvh) * g.max_seq;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(smem_u32(&full[s]), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  for (int c = threadIdx.x; c < RMAX * CPR; c += NT) {
    const int r = c / CPR, cc = c - r * CPR;
    const bool in = r < nrows;
    const bf16* src = in ? q + (size_t)(start + t0 + r / G) * g.ld_q + (kvh * G + r % G) * D + cc * 8 : q;
    cp_async16(smem_u32(Qs + r * LDQ + cc * 8), src, in);
  }
  cp_async_commit();
  __syncthreads();
  // With the in-kernel append, tiles below the first appended key are loaded while the append
  // runs; the rest wait for it.
  const int n_pre = app.on ? min(min(NS - 1, n_tiles), (pos0 + t0) / KT) : min(NS - 1, n_tiles);
  int n_issued = 0;                     // thread 0: key tiles issued so far (in tile order)
  auto issue = [&](int tile) {
    n_issued = tile + 1;
    const int s = tile % NS;
    const uint32_t fb = smem_u32(&full[s]);
    const uint32_t dst = smem_u32(stages + s * STAGE);
    mbar_arrive_expect_tx(fb, STAGE);
#pragma unroll
    for (int h = 0; h < HALVES; ++h) {
      tma_load_2d(dst + h * SUB, &kmap, h * 64, crow + tile * KT, fb);
      tma_load_2d(dst + (HALVES + h) * SUB, &vmap, h * 64, crow + tile * KT, fb);
    }
  };
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
    for (int t = 0; t < n_pre; ++t) issue(t);
  }
  if (app.on) {
    // RoPE (rotate-half, reference bf16 roundings as in the rope/KV kernel) and the KV append for
    // this item's tokens, in one pass: every global load (k, v, cos, sin) is issued while the Q rows
    // land by cp.async; after one barrier each thread rotates its (token, pair) of k and writes it to
    // the cache, writes its v chunk, and rotates the same pair of the token's G query rows in shared
    // memory with the same cos / sin.  The proxy fence orders the cache stores before the TMA reads of
    // those key tiles, which are issued only after the second barrier.
    const int half = D / 2;
    const bool valid = row >= 0 && row < g.max_batch && pos0 >= 0 && pos0 + t0 + nt <= g.max_seq;
    if (!valid && threadIdx.x == 0) set_status(status, kStatusBadIndex);
    bf16* kc = static_cast<bf16*>(app.kc) + ((size_t)row * g.n_kv_heads + kvh) * g.max_seq * D;
    bf16* vc = static_cast<bf16*>(app.vc) + ((size_t)row * g.n_kv_heads + kvh) * g.max_seq * D;
    constexpr int kU = 4;     // (token, pair) items per thread and pass
    constexpr int kV = 2;     // 16-byte v chunks per thread and pass
    const int n_k = valid ? nt * half : 0, n_v = valid ? nt * (D / 8) : 0;
    const int passes = max((n_k + kU * NT - 1) / (kU * NT), (n_v + kV * NT - 1) / (kV * NT));   // same on every thread
    for (int ps = 0; ps < passes; ++ps) {
      float x1[kU], x2[kU], c1[kU], c2[kU], s1[kU], s2[kU];
      uint4 vv[kV];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int i = threadIdx.x + (ps * kU + u) * NT;
        if (i < n_k) {
          const int tt = i / half, d = i - tt * half, pos = pos0 + t0 + tt;
          const bf16* src = q + (size_t)(start + t0 + tt) * g.ld_q + (g.n_heads + kvh) * D;
          x1[u] = __bfloat162float(__ldg(src + d));
          x2[u] = __bfloat162float(__ldg(src + d + half));
          c1[u] = __ldg(app.cos + (size_t)pos * D + d);
          c2[u] = __ldg(app.cos + (size_t)pos * D + d + half);
          s1[u] = __ldg(app.sin + (size_t)pos * D + d);
          s2[u] = __ldg(app.sin + (size_t)pos * D + d + half);
        }
      }
#pragma unroll
      for (int u = 0; u < kV; ++u) {
        const int i = threadIdx.x + (ps * kV + u) * NT;
        if (i < n_v) {
          const int tt = i / (D / 8), c8 = i - tt * (D / 8);
          vv[u] = __ldg(reinterpret_cast<const uint4*>(q + (size_t)(start + t0 + tt) * g.ld_q +
                                                       (g.n_heads + g.n_kv_heads + kvh) * D) + c8);
        }
      }
      if (ps == 0) {            // the Q rows (every thread's cp.async) are in shared memory after this
        cp_async_wait<0>();
        __syncthreads();
      }
#pragma unroll
      for (int u = 0; u < kV; ++u) {
        const int i = threadIdx.x + (ps * kV + u) * NT;
        if (i < n_v) {
          const int tt = i / (D / 8), c8 = i - tt * (D / 8);
          reinterpret_cast<uint4*>(vc + (size_t)(pos0 + t0 + tt) * D)[c8] = vv[u];
        }
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int i = threadIdx.x + (ps * kU + u) * NT;
        if (i < n_k) {
          const int tt = i / half, d = i - tt * half, pos = pos0 + t0 + tt;
          const float cc1 = rnd<bf16>(c1[u]), cc2 = rnd<bf16>(c2[u]), ss1 = rnd<bf16>(s1[u]), ss2 = rnd<bf16>(s2[u]);
          const float k1 = rnd<bf16>(x1[u] * cc1) + rnd<bf16>(-x2[u] * ss1);
          const float k2 = rnd<bf16>(x2[u] * cc2) + rnd<bf16>(x1[u] * ss2);
          kc[(size_t)pos * D + d] = __float2bfloat16_rn(k1);
          kc[(size_t)pos * D + d + half] = __float2bfloat16_rn(k2);
          for (int gh = 0; gh < G; ++gh) {          // the token's G query rows (disjoint per thread)
            bf16* qr = Qs + (tt * G + gh) * LDQ;
            const float y1 = __bfloat162float(qr[d]), y2 = __bfloat162float(qr[d + half]);
            qr[d] = __float2bfloat16_rn(rnd<bf16>(y1 * cc1) + rnd<bf16>(-y2 * ss1));
            qr[d + half] = __float2bfloat16_rn(rnd<bf16>(y2 * cc2) + rnd<bf16>(y1 * ss2));
          }
        }
      }
    }
    if (passes == 0) {          // nothing to append (an invalid block): Q still has to land
      cp_async_wait<0>();
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __syncthreads();
    // the tiles holding the appended keys go out only now
    if (threadIdx.x == 0)
      for (int t = n_pre; t < NS - 1 && t < n_tiles; ++t) issue(t);
  } else {
    cp_async_wait<0>();
    __syncthreads();
  }

  const int gq = lane >> 2, tq = lane & 3;
  const int n_rg = (nrows + 15) / 16;                   // row groups with rows
  const int rg = warp >> 2;                             // this warp's row group
  const int kq = warp & 3;                              // this warp's key quarter
  int qpos[2];
  {
    const int r0 = rg * 16 + gq, r1 = r0 + 8;
    qpos[0] = r0 < nrows ? pos0 + t0 + r0 / G : -1;
    qpos[1] = r1 < nrows ? pos0 + t0 + r1 / G : -1;
  }
  float o[ND][4];
  float m[2], l[2];
  m[0] = m[1] = -INFINITY;
  l[0] = l[1] = 0.f;
#pragma unroll
  for (int n = 0; n < ND; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  const int kw = kq * 16;                               // this warp's keys inside every tile
  const float scale_l2 = g.scale * 1.4426950408889634f;  // softmax scale times log2(e)

  for (int tile = 0; tile < n_tiles; ++tile) {
    if (threadIdx.x == 0 && tile + NS - 1 < n_tiles) issue(tile + NS - 1);
    if (!mbar_wait(smem_u32(&full[tile % NS]), (tile / NS) & 1, abort_flag, g.spin)) {
      set_status(status, kStatusTimeoutMma);
      *abort_flag = 1;
    }
    const uint32_t kt = smem_u32(stages + (tile % NS) * STAGE);
    const uint32_t vt = kt + HALVES * SUB;
    {
      if (rg < n_rg) {
        float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
          ldsm_x4(smem_u32(Qs + (rg * 16 + (lane & 15)) * LDQ + kk * 16 + (lane >> 4) * 8), a0, a1, a2, a3);
          const int key = kw + (lane & 7) + ((lane >> 4) << 3);
          const int dim = kk * 16 + ((lane >> 3) & 1) * 8;
          const uint32_t chunk = (uint32_t)((dim & 63) >> 3) ^ (uint32_t)(key & 7);
          ldsm_x4(kt + (dim >> 6) * SUB + key * 128 + chunk * 16, b0, b1, b2, b3);
          mma_bf16(s[0], a0, a1, a2, a3, b0, b1);
          mma_bf16(s[1], a0, a1, a2, a3, b2, b3);
        }
        // scores in the log2 domain (scale * log2 e folded in); only tiles reaching past the
        // item's first query position need the causal mask
        const int kbase = tile * KT + kw + 2 * tq;
        const bool need_mask = tile * KT + kw + 15 > pos0 + t0;
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int n = 0; n < 2; ++n) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            s[n][e] *= scale_l2;
            s[n][2 + e] *= scale_l2;
            if (need_mask) {
              const int key = kbase + n * 8 + e;
              if (key > qpos[0]) s[n][e] = -INFINITY;
              if (key > qpos[1]) s[n][2 + e] = -INFINITY;
            }
            mx0 = fmaxf(mx0, s[n][e]);
            mx1 = fmaxf(mx1, s[n][2 + e]);
          }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m[0], mx0), mn1 = fmaxf(m[1], mx1);
        // the running output needs rescaling only when some row's maximum moved
        const bool moved = !__all_sync(0xffffffffu, mn0 == m[0] && mn1 == m[1]);
        const float ms0 = mn0 == -INFINITY ? 0.f : mn0, ms1 = mn1 == -INFINITY ? 0.f : mn1;
        const float c0 = fast_exp2(m[0] - ms0), c1 = fast_exp2(m[1] - ms1);
        m[0] = mn0;
        m[1] = mn1;
        float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
        for (int n = 0; n < 2; ++n) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            s[n][e] = fast_exp2(s[n][e] - ms0);
            s[n][2 + e] = fast_exp2(s[n][2 + e] - ms1);
            ps0 += s[n][e];
            ps1 += s[n][2 + e];
          }
        }
        l[0] = l[0] * c0 + ps0;
        l[1] = l[1] * c1 + ps1;
        const uint32_t p0 = pack_bf16(s[0][0], s[0][1]), p1 = pack_bf16(s[0][2], s[0][3]);
        const uint32_t p2 = pack_bf16(s[1][0], s[1][1]), p3 = pack_bf16(s[1][2], s[1][3]);
        if (moved) {
#pragma unroll
          for (int n = 0; n < ND; ++n) {
            o[n][0] *= c0;
            o[n][1] *= c0;
            o[n][2] *= c1;
            o[n][3] *= c1;
          }
        }
#pragma unroll
        for (int n2 = 0; n2 < ND; n2 += 2) {
          const int key = kw + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int dim = n2 * 8 + (lane >> 4) * 8;
          const uint32_t chunk = (uint32_t)((dim & 63) >> 3) ^ (uint32_t)(key & 7);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(vt + (dim >> 6) * SUB + key * 128 + chunk * 16, b0, b1, b2, b3);
          mma_bf16(o[n2], p0, p1, p2, p3, b0, b1);
          mma_bf16(o[n2 + 1], p0, p1, p2, p3, b2, b3);
        }
      }
    }
    __syncthreads();
    if (*abort_flag) break;   // set before this barrier only, so every thread leaves together
  }
  if (*abort_flag) {
    // A wait gave up: no tile is issued after it, and every stage holds at most one outstanding
    // load (a stage is refilled only after its previous tile was waited for), so waiting for the
    // last tile issued into each stage lets every copy land before the CTA exits.
    if (threadIdx.x == 0)
      for (int st = 0; st < NS && st < n_issued; ++st) {
        const int last = st + (n_issued - 1 - st) / NS * NS;
        mbar_drain(smem_u32(&full[st]), (uint32_t)(last / NS) & 1u);
      }
    __syncthreads();
    return;
  }
  // ---- merge the four key quarters' partial states in quarter order (stage memory is free now)
  constexpr int OLD = D + 4;
  float* Ms = reinterpret_cast<float*>(stages);          // [4][RMAX]
  float* Lw = Ms + 4 * RMAX;                             // [4][RMAX]
  float* Ow = Lw + 4 * RMAX;                             // [4][RMAX][OLD]
  static_assert((8 * RMAX + 4 * RMAX * (D + 4)) * 4 <= NS * STAGE, "merge buffers exceed the stage memory");
  if (rg < n_rg) {
    float l0 = l[0], l1 = l[1];
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const int r0 = rg * 16 + gq, r1 = r0 + 8;
    if (tq == 0) {
      Ms[kq * RMAX + r0] = m[0];
      Ms[kq * RMAX + r1] = m[1];
      Lw[kq * RMAX + r0] = l0;
      Lw[kq * RMAX + r1] = l1;
    }
#pragma unroll
    for (int n = 0; n < ND; ++n) {
      const int d = n * 8 + 2 * tq;
      *reinterpret_cast<float2*>(&Ow[(kq * RMAX + r0) * OLD + d]) = make_float2(o[n][0], o[n][1]);
      *reinterpret_cast<float2*>(&Ow[(kq * RMAX + r1) * OLD + d]) = make_float2(o[n][2], o[n][3]);
    }
  }
  __syncthreads();
  const int hd = g.n_heads * D;
  for (int idx = threadIdx.x; idx < nrows * (D / 2); idx += NT) {
    const int r = idx / (D / 2), d = (idx - r * (D / 2)) * 2;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) mx = fmaxf(mx, Ms[w * RMAX + r]);
    float lsum = 0.f, a = 0.f, bsum = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = Ms[w * RMAX + r];
      const float f = mw == -INFINITY ? 0.f : fast_exp2(mw - mx);
      const float2 ov = *reinterpret_cast<const float2*>(&Ow[(w * RMAX + r) * OLD + d]);
      lsum += Lw[w * RMAX + r] * f;
      a += ov.x * f;
      bsum += ov.y * f;
    }
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
    bf16* p = out + (size_t)(start + t0 + r / G) * hd + (kvh * G + r % G) * D + d;
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a * inv, bsum * inv);
  }
}

// ---------------------------------------------------------------- small step kernels
template <typename T>
__global__ void embed_kernel(const T* __restrict__ table, const int32_t* __restrict__ ids, int dim, int vocab,
                             T* __restrict__ x, int* status) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x;
  const int id = ids[i];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) set_status(status, kStatusBadIndex);
    for (int j = threadIdx.x; j < dim; j += blockDim.x) x[(size_t)i * dim + j] = from_f<T>(0.f);
    return;
  }
  for (int j = threadIdx.x; j < dim; j += blockDim.x) x[(size_t)i * dim + j] = table[(size_t)id * dim + j];
}

__global__ void copy_rows_kernel(const uint8_t* __restrict__ src, const int32_t* __restrict__ si, uint8_t* __restrict__ dst,
                                 const int32_t* __restrict__ di, int row_bytes) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x;
  const uint8_t* s = src + (size_t)(si ? si[i] : i) * row_bytes;
  uint8_t* d = dst + (size_t)(di ? di[i] : i) * row_bytes;
  if ((row_bytes & 15) == 0 && ((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d)) & 15) == 0) {
    for (int j = threadIdx.x; j < row_bytes / 16; j += blockDim.x)
      reinterpret_cast<uint4*>(d)[j] = reinterpret_cast<const uint4*>(s)[j];
  } else {
    for (int j = threadIdx.x; j < row_bytes; j += blockDim.x) d[j] = s[j];
  }
}

__global__ void gather_ids_kernel(const int32_t* __restrict__ table, const int32_t* __restrict__ idx,
                                  int32_t* __restrict__ ids, int n) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) ids[i] = table[idx[i]];
}
__global__ void scatter_ids_kernel(const int32_t* __restrict__ ids, const int32_t* __restrict__ idx,
                                   int32_t* __restrict__ table, int n) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) table[idx[i]] = ids[i];
}

// Greedy acceptance: first mismatch between the verified tokens and the drafts; the token at
// that position (the correction, or the bonus token when all drafts match) becomes the
// verifier's next input (solutions/engine.py:464-475).
__global__ void greedy_accept_kernel(const int32_t* __restrict__ y, const int32_t* __restrict__ vinfo, int nv,
                                     int32_t* __restrict__ seq_buf, int stride, int32_t* __restrict__ acc) {
  pdl_trigger();
  pdl_wait();
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= nv) return;
  const int start = vinfo[3 * v], T = vinfo[3 * v + 1], slot = vinfo[3 * v + 2];
  int32_t* sb = seq_buf + (size_t)slot * stride;
  int a = 0;
  while (a < T - 1 && y[start + a] == sb[a + 1]) ++a;
  acc[v] = a;
  sb[0] = y[start + a];
}

// Packed metadata of one draft/verify round, built on the device from the round-start positions
// (the host does not wait for the previous round's acceptance).  Thread (i, t): request i of the
// active list, token t of its round; layout in round_meta_ints().
__global__ void round_meta_kernel(const int32_t* __restrict__ act, int n, const int32_t* __restrict__ pos,
                                  int max_batch, int cols, int item_tokens, int32_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * cols) return;
  const int i = idx / cols, t = idx - i * cols;
  const int slot = act[i];
  const int p0 = (slot >= 0 && slot < max_batch) ? pos[slot] : 0;
  // shallow step t: token t of every request, one token per block
  int32_t* st = out + (size_t)t * 10 * n;
  st[i] = p0 + t;                                   // tok_pos
  st[n + i] = slot;                                 // tok_row
  st[2 * n + 4 * i] = i;                            // blk (start, T, row, pos0)
  st[2 * n + 4 * i + 1] = 1;
  st[2 * n + 4 * i + 2] = slot;
  st[2 * n + 4 * i + 3] = p0 + t;
  st[6 * n + 2 * i] = i;                            // items (block, first token)
  st[6 * n + 2 * i + 1] = 0;
  st[8 * n + i] = slot * cols + t;                  // seq_buf / exit_h row of the token
  st[9 * n + i] = slot * cols + t + 1;              // seq_buf cell of its draft
  // verify step: all cols tokens of every request
  const int ni = (cols + item_tokens - 1) / item_tokens;
  int32_t* v = out + (size_t)cols * 10 * n;
  const int nt = n * cols;
  v[i * cols + t] = p0 + t;                         // tok_pos
  v[nt + i * cols + t] = slot;                      // tok_row
  int32_t* vblk = v + 2 * nt;
  int32_t* vitems = vblk + 4 * n;
  int32_t* vrows = vitems + 2 * n * ni;
  int32_t* vinfo = vrows + nt;
  vrows[i * cols + t] = slot * cols + t;
  if (t == 0) {
    vblk[4 * i] = i * cols;
    vblk[4 * i + 1] = cols;
    vblk[4 * i + 2] = slot;
    vblk[4 * i + 3] = p0;
    for (int k = 0; k < ni; ++k) {
      vitems[2 * (i * ni + k)] = i;
      vitems[2 * (i * ni + k) + 1] = k * item_tokens;
    }
    vinfo[3 * i] = i * cols;
    vinfo[3 * i + 1] = cols;
    vinfo[3 * i + 2] = slot;
  }
}

// Round-start positions of the next round: every request advances by its accepted drafts + 1.
__global__ void round_advance_kernel(const int32_t* __restrict__ act, int n, const int32_t* __restrict__ acc,
                                     int32_t* __restrict__ pos, int max_batch) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int slot = act[i];
  if (slot >= 0 && slot < max_batch) pos[slot] += acc[i] + 1;
}

// argmax keys -> token ids.  With a status word: a non-zero word (a timed-out wait or a bad row in
// the kernels before) turns every id into -1, and the word is copied to status_out (nullable).
__global__ void keys_to_ids_kernel(const unsigned long long* __restrict__ keys, int32_t* __restrict__ ids, int n,
                                   const int* status, int32_t* status_out) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int st = status ? *(volatile const int*)status : 0;
  if (i == 0 && status_out) *status_out = st;
  if (i < n) ids[i] = st ? -1 : (int32_t)(0xFFFFFFFFu - (uint32_t)(keys[i] & 0xFFFFFFFFull));
}

// argmax over logits rows (lowest index on ties, as torch.argmax)
template <typename T>
__global__ void __launch_bounds__(256) argmax_rows_kernel(const T* __restrict__ logits, int vocab, int32_t* __restrict__ ids) {
  pdl_trigger();
  pdl_wait();
  __shared__ unsigned long long red[8];
  const int i = blockIdx.x;
  const T* lr = logits + (size_t)i * vocab;
  unsigned long long best = 0;
  for (int j = threadIdx.x; j < vocab; j += 256) {
    const unsigned long long k = argmax_key(to_f(lr[j]), (uint32_t)j);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
    best = v > best ? v : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; ++w) best = red[w] > best ? red[w] : best;
    best = red[0] > best ? red[0] : best;
    ids[i] = (int32_t)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
  }
}

__global__ void swiglu_f32_kernel(const float* __restrict__ gu, float* __restrict__ out, int n, int inter) {
  pdl_trigger();
  pdl_wait();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)n * inter) return;
  const size_t t = i / inter, j = i - t * inter;
  const float g = gu[t * 2 * inter + j], u = gu[t * 2 * inter + inter + j];
  out[i] = g / (1.0f + expf(-g)) * u;
}

// fp32 CUDA-core GEMM (parity path): 64 x 64 tiles, 16-wide K steps, 4 x 4 outputs per thread.
// Each output is a sequential fp32 sum over K, independent of the token count.
__global__ void __launch_bounds__(256) simt_gemm_f32_kernel(int epi, const float* __restrict__ x,
                                                            const float* __restrict__ w, const float* residual,
                                                            float* y, int n_tok, int n_out, int K) {
  pdl_trigger();
  pdl_wait();
  __shared__ float As[16][68];
  __shared__ float Bs[16][68];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int t0 = blockIdx.y * 64, o0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int idx = threadIdx.x; idx < 64 * 16; idx += 256) {
      const int r = idx >> 4, kk = idx & 15;
      const int k = k0 + kk;
      As[kk][r] = (t0 + r < n_tok && k < K) ? x[(size_t)(t0 + r) * K + k] : 0.f;
      Bs[kk][r] = (o0 + r < n_out && k < K) ? w[(size_t)(o0 + r) * K + k] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], bb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = As[kk][ty * 4 + i];
        bb[i] = Bs[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + ty * 4 + i;
    if (t >= n_tok) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int o = o0 + tx * 4 + j;
      if (o >= n_out) continue;
      const size_t idx = (size_t)t * n_out + o;
      y[idx] = epi == EESD_EPI_RESIDUAL ? residual[idx] + acc[i][j] : acc[i][j];
    }
  }
}

inline int launched() { return cudaPeekAtLastError() == cudaSuccess ? EESD_OK : EESD_ERR_CUDA; }

}  // namespace

int attn_item_tokens(int n_heads, int n_kv_heads) {
  const int G = n_heads / n_kv_heads;
  return G >= 32 ? 1 : 32 / G;   // up to 32 query rows per work item
}

int launch_rmsnorm(int dtype, const void* x, const int32_t* rows, const void* w, void* y, int n, int dim, float eps,
                   cudaStream_t s, int n_src, int* status) {
  if (n <= 0) return EESD_OK;
  if (dtype == EESD_BF16)
    launch_pdl(rmsnorm_kernel<bf16>, dim3(n), dim3(256), 0, s, (const bf16*)x, rows, (const bf16*)w, (bf16*)y, dim, eps,
               n_src, status);
  else
    launch_pdl(rmsnorm_kernel<float>, dim3(n), dim3(256), 0, s, (const float*)x, rows, (const float*)w, (float*)y, dim,
               eps, n_src, status);
  return launched();
}

int launch_rope_kv(int dtype, void* qkv, const int32_t* tok_pos, const int32_t* tok_row, int n_tok, int n_heads,
                   int n_kv_heads, int head_dim, const float* cos, const float* sin, void* kc, void* vc, int max_batch,
                   int max_seq, int* status, cudaStream_t s) {
  if (n_tok <= 0) return EESD_OK;
  if (dtype == EESD_BF16)
    launch_pdl(rope_kv_kernel<bf16>, dim3(n_tok), dim3(256), 0, s, (bf16*)qkv, tok_pos, tok_row, n_heads, n_kv_heads, head_dim, cos, sin,
                                               (bf16*)kc, (bf16*)vc, max_batch, max_seq, status);
  else
    launch_pdl(rope_kv_kernel<float>, dim3(n_tok), dim3(256), 0, s, (float*)qkv, tok_pos, tok_row, n_heads, n_kv_heads, head_dim, cos, sin,
                                                (float*)kc, (float*)vc, max_batch, max_seq, status);
  return launched();
}

template <int D, int WARPS, int NS, int MINB>
int launch_attn_variant(dim3 grid, cudaStream_t s, const CUtensorMap& kmap, const CUtensorMap& vmap, const AttnGeom& g,
                        int it, int layer, const void* q, void* out, const int32_t* blk, const int32_t* items,
                        int* status, const AttnAppend& app) {
  constexpr int RMAX = 16 * (WARPS / 4);
  const size_t sm = 1024 + (size_t)NS * (2 * (D / 64) * 64 * 128) + (size_t)RMAX * (D + 8) * 2 + 64;
  static bool set = false;
  if (!set) {
    if (cudaFuncSetAttribute(attn_bf16_kernel<D, WARPS, NS, MINB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sm))
      return EESD_ERR_CUDA;
    set = true;
  }
  launch_pdl(attn_bf16_kernel<D, WARPS, NS, MINB>, grid, dim3(WARPS * 32), sm, s, kmap, vmap, g, it, layer,
             (const bf16*)q, (bf16*)out, blk, items, status, app);
  return EESD_OK;
}

int launch_attention(int dtype, const AttnGeom& g_in, const void* q, const void* kc, const void* vc, void* out,
                     const int32_t* blk, const int32_t* items, int n_items, int max_ctx, int* status, cudaStream_t s,
                     const CUtensorMap* kmap, const CUtensorMap* vmap, int layer, const AttnAppend& app,
                     int rows_max) {
  (void)max_ctx;
  if (app.on && (dtype != EESD_BF16 || !app.kc || !app.vc || !app.cos || !app.sin)) return EESD_ERR_ARG;
  if (n_items <= 0) return EESD_OK;
  const int it = attn_item_tokens(g_in.n_heads, g_in.n_kv_heads);
  AttnGeom g = g_in;
  g.status = status;
  g.spin = spin_limit();
  g.n_items = n_items;
  dim3 grid(n_items, g.n_kv_heads);
  if (dtype == EESD_BF16) {
    if (!kmap || !vmap || n_items > 65535) return EESD_ERR_ARG;
    grid = dim3(g.n_kv_heads, n_items);
    // rows per item <= 16: 4 warps, 2 stages, 3 CTAs per SM; else 8 warps, 3 stages, 2 per SM
    const bool small = rows_max <= 16;
    int rc;
    if (g.head_dim == 128)
      rc = small ? launch_attn_variant<128, 4, 2, 3>(grid, s, *kmap, *vmap, g, it, layer, q, out, blk, items, status, app)
                 : launch_attn_variant<128, 8, 3, 2>(grid, s, *kmap, *vmap, g, it, layer, q, out, blk, items, status, app);
    else if (g.head_dim == 64)
      rc = small ? launch_attn_variant<64, 4, 2, 3>(grid, s, *kmap, *vmap, g, it, layer, q, out, blk, items, status, app)
                 : launch_attn_variant<64, 8, 3, 2>(grid, s, *kmap, *vmap, g, it, layer, q, out, blk, items, status, app);
    else
      return EESD_ERR_ARG;
    if (rc) return rc;
  } else {
    const size_t layer_off = (size_t)g.max_batch * g.n_kv_heads * g.max_seq * g.head_dim * (size_t)layer;
    const float* kl = static_cast<const float*>(kc) + layer_off;
    const float* vl = static_cast<const float*>(vc) + layer_off;
    if (g.head_dim == 128) {
      const size_t sm = (size_t)(32 * 128 + 32 * 129 + 32 * 128) * 4;
      static bool set = false;
      if (!set) {
        if (cudaFuncSetAttribute(attn_f32_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm))
          return EESD_ERR_CUDA;
        set = true;
      }
      launch_pdl(attn_f32_kernel<128>, dim3(grid), dim3(128), sm, s, g, it, (const float*)q, kl, vl, (float*)out, blk, items);
    } else if (g.head_dim == 64) {
      const size_t sm = (size_t)(32 * 64 + 32 * 65 + 32 * 64) * 4;
      launch_pdl(attn_f32_kernel<64>, dim3(grid), dim3(128), sm, s, g, it, (const float*)q, kl, vl, (float*)out, blk, items);
    } else {
      return EESD_ERR_ARG;
    }
  }
  return launched();
}

// One CTA: item i's slot is the number of items that run before it (more keys, or as many keys
// and a lower index), so the slots form a permutation whatever the lengths are.  An item whose
// block index is out of range sorts last; the attention kernel reports it.
__global__ void __launch_bounds__(1024) attn_order_kernel(const int32_t* __restrict__ blk,
                                                          const int32_t* __restrict__ items, int n_items, int n_blocks,
                                                          int item_tokens, int32_t* __restrict__ order) {
  pdl_trigger();
  pdl_wait();
  __shared__ int keys[kAttnOrderMax];
  for (int i = threadIdx.x; i < n_items; i += blockDim.x) {
    const int b = items[2 * i], t0 = items[2 * i + 1];
    int len = -1;
    if (b >= 0 && b < n_blocks) len = blk[4 * b + 3] + t0 + min(item_tokens, blk[4 * b + 1] - t0);
    keys[i] = len;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n_items; i += blockDim.x) {
    const int li = keys[i];
    int slot = 0;
    for (int k = 0; k < n_items; ++k) {
      const int lk = keys[k];
      slot += (lk > li) | ((lk == li) & (k < i));
    }
    order[slot] = i;
  }
}

int launch_attn_order(const int32_t* blk, const int32_t* items, int n_items, int n_blocks, int n_heads, int n_kv_heads,
                      int32_t* order, cudaStream_t s) {
  if (n_items <= 0) return EESD_OK;
  if (n_items > kAttnOrderMax) return EESD_ERR_ARG;
  launch_pdl(attn_order_kernel, dim3(1), dim3(1024), 0, s, blk, items, n_items, n_blocks,
             attn_item_tokens(n_heads, n_kv_heads), order);
  return launched();
}

int launch_embed(int dtype, const void* table, const int32_t* ids, int n, int dim, int vocab, void* x, int* status,
                 cudaStream_t s) {
  if (n <= 0) return EESD_OK;
  if (dtype == EESD_BF16)
    launch_pdl(embed_kernel<bf16>, dim3(n), dim3(256), 0, s, (const bf16*)table, ids, dim, vocab, (bf16*)x, status);
  else
    launch_pdl(embed_kernel<float>, dim3(n), dim3(256), 0, s, (const float*)table, ids, dim, vocab, (float*)x, status);
  return launched();
}

int launch_copy_rows(int dtype, const void* src, const int32_t* src_idx, void* dst, const int32_t* dst_idx, int n,
                     int width, cudaStream_t s) {
  if (n <= 0) return EESD_OK;
  const int eb = dtype == EESD_BF16 ? 2 : 4;
  launch_pdl(copy_rows_kernel, dim3(n), dim3(128), 0, s, (const uint8_t*)src, src_idx, (uint8_t*)dst, dst_idx, width * eb);
  return launched();
}

int launch_gather_ids(const int32_t* table, const int32_t* idx, int32_t* ids, int n, cudaStream_t s) {
  if (n <= 0) return EESD_OK;
  launch_pdl(gather_ids_kernel, dim3((n + 255) / 256), dim3(256), 0, s, table, idx, ids, n);
  return launched();
}
int launch_scatter_ids(const int32_t* ids, const int32_t* idx, int32_t* table, int n, cudaStream_t s) {
  if (n <= 0) return EESD_OK;
  launch_pdl(scatter_ids_kernel, dim3((n + 255) / 256), dim3(256), 0, s, ids, idx, table, n);
  return launched();
}
int launch_greedy_accept(const int32_t* y, const int32_t* vinfo, int nv, int32_t* seq_buf, int stride, int32_t* acc,
                         cudaStream_t s) {
  if (nv <= 0) return EESD_OK;
  launch_pdl(greedy_accept_kernel, dim3((nv + 127) / 128), dim3(128), 0, s, y, vinfo, nv, seq_buf, stride, acc);
  return launched();
}
int launch_round_meta(const int32_t* act, int n, const int32_t* pos, int max_batch, int cols, int item_tokens,
                      int32_t* out, cudaStream_t s) {
  if (n <= 0) return EESD_OK;
  launch_pdl(round_meta_kernel, dim3((n * cols + 127) / 128), dim3(128), 0, s, act, n, pos, max_batch, cols,
             item_tokens, out);
  return launched();
}
int launch_round_advance(const int32_t* act, int n, const int32_t* acc, int32_t* pos, int max_batch, cudaStream_t s) {
  if (n <= 0) return EESD_OK;
  launch_pdl(round_advance_kernel, dim3((n + 127) / 128), dim3(128), 0, s, act, n, acc, pos, max_batch);
  return launched();
}
int launch_keys_to_ids(const unsigned long long* keys, int32_t* ids, int n, cudaStream_t s, const int* status,
                       int32_t* status_out) {
  if (n <= 0) return EESD_OK;
  launch_pdl(keys_to_ids_kernel, dim3((n + 255) / 256), dim3(256), 0, s, keys, ids, n, status, status_out);
  return launched();
}
int launch_argmax_rows(int dtype, const void* logits, int n, int vocab, int32_t* ids, cudaStream_t s) {
  if (n <= 0) return EESD_OK;
  if (dtype == EESD_BF16)
    launch_pdl(argmax_rows_kernel<bf16>, dim3(n), dim3(256), 0, s, (const bf16*)logits, vocab, ids);
  else
    launch_pdl(argmax_rows_kernel<float>, dim3(n), dim3(256), 0, s, (const float*)logits, vocab, ids);
  return launched();
}
int launch_swiglu_f32(const float* gu, float* out, int n, int inter, cudaStream_t s) {
  if (n <= 0) return EESD_OK;
  const size_t tot = (size_t)n * inter;
  launch_pdl(swiglu_f32_kernel, dim3((unsigned)((tot + 255) / 256)), dim3(256), 0, s, gu, out, n, inter);
  return launched();
}
int launch_simt_gemm_f32(int epi, const float* x, const float* w, const float* residual, float* y, int n_tok, int n_out,
                         int k, cudaStream_t s) {
  if (n_tok <= 0) return EESD_OK;
  dim3 grid((n_out + 63) / 64, (n_tok + 63) / 64);
  launch_pdl(simt_gemm_f32_kernel, dim3(grid), dim3(256), 0, s, epi, x, w, residual, y, n_tok, n_out, k);
  return launched();
}

}  // namespace eesd
