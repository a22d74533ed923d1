// tcgen05 / TMEM bf16 GEMM for the packed token axis:  Y[t, o] = epi( sum_k X[t, k] * W[o, k] ).
//
// Replaces the F.linear calls of solutions/packed.py:175-185 (QKV, O + residual, W13 + SwiGLU,
// W2 + residual) and the LM head of common/model.py:328-330 (+ argmax).
//
// Mapping: the weight is the MMA "A" operand (M = 128 output features per CTA), the packed
// tokens are "B" (N = token tile, <= 256), both K-major in shared memory with 128-byte
// swizzle, staged by TMA; the fp32 accumulator lives in TMEM (128 lanes x N columns).
//   warp 0      TMA producer (one elected lane), STAGES-deep ring of (W tile, X tile)
//   warp 1      TMEM allocator + MMA issuer (one lane), tcgen05.commit frees a stage
//   warps 2..9  epilogue: two warps per 32-lane TMEM quadrant (warp % 4), alternating 16-column
//               chunks; tcgen05.ld, fused epilogue, stores
// Token tiles are up to 256 tokens for SwiGLU (two accumulators) and 384 otherwise; a tile wider
// than 256 is fed by two TMA boxes and two MMAs per k-step.
// SwiGLU keeps two accumulators (gate rows o and up rows o + I) in the same TMEM lanes, so
// silu(g) * u is formed per thread with no data exchange.
//
// Split-K (few output tiles, e.g. the O and W2 projections): the S CTAs that share an output
// tile form one thread-block cluster (1 x 1 x S).  After the main loop each CTA stores the fp32
// partial sums of the token columns it does not own to a global (L2-resident) scratch, one
// cluster barrier publishes them, and CTA r sums column slice r over the S splits in split
// order, then applies the epilogue.
//
// Batch invariance (needed for bit-exact speculative == autoregressive output): the K range
// of every split and the split count depend only on the weight shape, the split sum has a
// fixed order, and every token column is an independent dot product (checked on hardware for
// every MMA N).  No atomics touch values except the order-free argmax max().
#include <algorithm>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "gemm_tc.h"

namespace eesd {

namespace {

constexpr int kBM = 128;   // output features per CTA (MMA M)
constexpr int kBK = 64;    // K per stage: 64 bf16 = one 128-byte swizzle row
constexpr int kThreads = 320;
constexpr int kEpiThreads = 256;           // warps 2..9
constexpr uint32_t kATileBytes = kBM * kBK * 2;
constexpr size_t kSmemBudget = 224 * 1024;
constexpr int kMaxSplits = 8;              // portable cluster size

struct alignas(8) TcParams {
  int n_tok, n_out, K;
  int bn;           // token tile (multiple of mma_n)
  int b_boxes;      // TMA boxes per token tile (1, or 2 of bn / 2 rows)
  int mma_n;        // N of one tcgen05.mma (multiple of 16, <= 256)
  int kb_total;     // ceil(K / 64)
  int kb_per;       // k-blocks per split
  int splits;       // = cluster size along z
  int stages;
  int up_offset;    // SwiGLU: row of the first 'up' weight
  int tmem_cols;
  int a_packed;     // 1: weight in tile-packed layout (3-D map over 16 KB tiles), 0: row-major 2-D map
  int acc_cols;     // TMEM columns of the accumulator (bn, or 2 bn for SwiGLU)
  int res_stage;    // split-K RESIDUAL: the owned slice's residual rows arrive by bulk copies (256 B each)
  int mma_n1;       // > 0: two MMAs per k-step, N = mma_n1 then bn - mma_n1 (token tiles above 256)
  const bf16* residual;
  int ld_res;
  bf16* y;
  int ld_y;
  unsigned long long* keys;  // argmax keys [n_tok]
  float4* partials;          // split-K: [tile][split][acc_cols / 4][128] fp32 partial tiles
  int* status;
  uint32_t spin;             // poll limit of the pipeline waits (spin_limit())
};

// named barrier of the 256 epilogue threads (bar.sync counts whole warps: converge first)
__device__ __forceinline__ void epi_bar() {
  __syncwarp();
  asm volatile("bar.sync 1, 256;" ::: "memory");
}
// silu(x) = x / (1 + exp(-x)) with the fast exponential and division (results are rounded to bf16)
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// Epilogue of NC consecutive token columns t0.. of one output row.  Residual values are all loaded
// before any store (the residual may be the output buffer itself, so interleaving would serialise
// every load behind the previous store).
template <int EPI, int NC>
__device__ __forceinline__ void load_residual(const TcParams& p, int t0, int row, float* r) {
  if (EPI == EESD_EPI_RESIDUAL) {
#pragma unroll
    for (int j = 0; j < NC; ++j)
      r[j] = (t0 + j < p.n_tok) ? __bfloat162float(p.residual[(size_t)(t0 + j) * p.ld_res + row]) : 0.f;
  }
}

// Epilogue with the residual values already loaded (r, RESIDUAL only)
template <int EPI, int NC>
__device__ __forceinline__ void epilogue_cols_r(const TcParams& p, int t0, int row, const float* g, const float* u,
                                                const float* r) {
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    const int t = t0 + j;
    if (t >= p.n_tok) break;
    const size_t o = (size_t)t * p.ld_y + row;
    if (EPI == EESD_EPI_STORE) {
      p.y[o] = __float2bfloat16_rn(g[j]);
    } else if (EPI == EESD_EPI_RESIDUAL) {
      // x + F.linear(...): the product is rounded to bf16 first, then the bf16 add rounds again
      p.y[o] = __float2bfloat16_rn(r[j] + rnd<bf16>(g[j]));
    } else if (EPI == EESD_EPI_SWIGLU) {
      // F.silu(g) * u in bf16: g, u rounded (F.linear output), silu rounded, product rounded
      const float gb = rnd<bf16>(g[j]), ub = rnd<bf16>(u[j]);
      p.y[o] = __float2bfloat16_rn(rnd<bf16>(silu_f(gb)) * ub);
    }
  }
}

template <int EPI, int NC>
__device__ __forceinline__ void epilogue_cols(const TcParams& p, int t0, int row, const float* g, const float* u) {
  float r[NC];
  load_residual<EPI, NC>(p, t0, row, r);
  epilogue_cols_r<EPI, NC>(p, t0, row, g, u, r);
}

// PAIR: a (2,1,1) cluster of two CTAs computes one 256-row x bn tile with cta_group::2 MMAs.  CTA r
// holds weight row tile 2 * blockIdx.z + r (its 128 accumulator lanes) and token rows
// [n0 + r bn/2, n0 + (r + 1) bn/2) of the tile; both CTAs' tile loads complete on the even CTA's
// `full` barriers, the even CTA alone issues the MMAs, and it commits to the `empty` and
// accumulator barriers of both CTAs (one commit per CTA).  Per SM, a k-block moves 128 weight rows and bn/2 token rows
// for 128 x bn outputs, where a single CTA moves 128 + bn rows.
template <int EPI, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x, TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // two A tiles per stage: SwiGLU (gate and up rows) and the two-tile head (rows m0 and m0 + 128)
  constexpr int kNA = (EPI == EESD_EPI_SWIGLU || EPI == EESD_EPI_ARGMAX2_INTERNAL) ? 2 : 1;
  const int b_rows = PAIR ? p.bn / 2 : p.bn;     // token rows this CTA loads per k-block
  const uint32_t b_bytes = (uint32_t)b_rows * kBK * 2;
  const uint32_t stage_bytes = kNA * kATileBytes + b_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)p.stages * stage_bytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + p.stages;
  uint64_t* accb = bars + 2 * p.stages;
  uint64_t* epib = accb + 1;                 // split-K: staged partials / residual landed
  uint64_t* drainb = accb + 2;               // after an abort: the MMAs already issued completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accb + 3);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = PAIR ? (int)cluster_rank() : 0;          // CTA of the pair (0 issues the MMAs)
  const int tok_tile = PAIR ? blockIdx.y : blockIdx.x;
  const int out_tile = PAIR ? 2 * blockIdx.z + rank : (EPI == EESD_EPI_ARGMAX2_INTERNAL ? 2 * blockIdx.y : blockIdx.y);
  const int split = PAIR ? 0 : blockIdx.z;
  const int n0 = tok_tile * p.bn, m0 = out_tile * kBM;
  const int kb_begin = split * p.kb_per;
  const int nkb = min(p.kb_total, kb_begin + p.kb_per) - kb_begin;
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(accb), 1);
    mbar_init(smem_u32(epib), 1);
    mbar_init(smem_u32(drainb), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_w);
    tma_prefetch_desc(&map_x);
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(smem_u32(tmem_slot), (uint32_t)p.tmem_cols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(tmem_slot), (uint32_t)p.tmem_cols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  // the pair's barriers and TMEM exist before either CTA signals the other
  if (PAIR) cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // what is in flight if the CTA aborts: k-blocks whose loads the producer issued, MMAs issued and
  // whether their completion was committed to the accumulator barrier (producer / issuer lanes)
  int loads_issued = 0;
  bool mma_issued = false, mma_committed = false;

  if (warp == 0) {
    if (lane == 0) {
      // Weight tiles do not depend on the previous kernel: the first stages' weight loads are issued
      // before waiting for it (programmatic dependent launch), the activation loads after.
      // fb: the `full` barrier that counts the load (PAIR: the even CTA's, as a cluster address)
      auto load_a = [&](int i, uint32_t st, uint32_t fb) {
        const int kb = kb_begin + i;
        if (p.a_packed) {
          // tile (row tile, k-block) = one contiguous 16 KB block: tiles of a row tile are consecutive
          const int z0 = out_tile * p.kb_total + kb, z1 = (out_tile + p.up_offset / kBM) * p.kb_total + kb;
          if (PAIR) {
            tma_load_3d_pair(st, &map_w, 0, 0, z0, fb);
            if (kNA == 2) tma_load_3d_pair(st + kATileBytes, &map_w, 0, 0, z1, fb);
          } else {
            tma_load_3d(st, &map_w, 0, 0, z0, fb);
            if (kNA == 2) tma_load_3d(st + kATileBytes, &map_w, 0, 0, z1, fb);
          }
        } else if (PAIR) {
          tma_load_2d_pair(st, &map_w, kb * kBK, m0, fb);
          if (kNA == 2) tma_load_2d_pair(st + kATileBytes, &map_w, kb * kBK, p.up_offset + m0, fb);
        } else {
          tma_load_2d(st, &map_w, kb * kBK, m0, fb);
          if (kNA == 2) tma_load_2d(st + kATileBytes, &map_w, kb * kBK, p.up_offset + m0, fb);
        }
      };
      auto load_b = [&](int i, uint32_t st, uint32_t fb) {
        const int kx = (kb_begin + i) * kBK;
        const uint32_t bst = st + kNA * kATileBytes;
        if (PAIR) {
          tma_load_2d_pair(bst, &map_x, kx, n0 + rank * b_rows, fb);
        } else {
          tma_load_2d(bst, &map_x, kx, n0, fb);
          if (p.b_boxes == 2) tma_load_2d(bst + (uint32_t)(p.bn / 2) * 128u, &map_x, kx, n0 + p.bn / 2, fb);
        }
      };
      // the even CTA of a pair expects both CTAs' bytes on its barrier; the odd CTA only loads
      const bool expects = !PAIR || rank == 0;
      const uint32_t tx_bytes = PAIR ? 2u * stage_bytes : stage_bytes;
      auto fbar = [&](int slot) {
        const uint32_t local = smem_u32(&full[slot]);
        return PAIR ? dsmem_addr(local, 0) : local;
      };
      const int pre = min(p.stages, nkb);
      for (int i = 0; i < pre; ++i) {
        if (expects) mbar_arrive_expect_tx(smem_u32(&full[i]), tx_bytes);
        load_a(i, smem_u32(smem + (size_t)i * stage_bytes), fbar(i));
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) load_b(i, smem_u32(smem + (size_t)i * stage_bytes), fbar(i));
      loads_issued = pre;
      const int stages = p.stages;
      const uint32_t smem0 = smem_u32(smem), empty0 = smem_u32(empty);
      int s = pre % stages, ph = (pre / stages) & 1;   // ring slot of k-block i and its fill parity
      for (int i = pre; i < nkb; ++i) {
        // slot s was last filled for k-block i - stages: wait for the MMAs that read it
        if (!mbar_wait(empty0 + 8u * s, ph ^ 1, abort_flag, p.spin)) {
          set_status(p.status, kStatusTimeoutProducer);
          *abort_flag = 1;
          break;
        }
        if (expects) mbar_arrive_expect_tx(smem_u32(&full[s]), tx_bytes);
        const uint32_t st = smem0 + (uint32_t)s * stage_bytes;
        const uint32_t fb = fbar(s);
        load_a(i, st, fb);
        load_b(i, st, fb);
        loads_issued = i + 1;
        if (++s == stages) { s = 0; ph ^= 1; }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && (!PAIR || rank == 0)) {
      // This single-thread loop is on the critical path (one tcgen05.mma per 4 KB of weights at
      // small token counts): loop-invariant values live in registers, descriptors are built once
      // per stage and stepped by adding to their 14-bit start-address field (bytes / 16).
      const uint32_t idesc = idesc_bf16_f32(PAIR ? 2 * kBM : kBM, p.mma_n);
      const uint32_t idesc1 = idesc_bf16_f32(kBM, p.mma_n1 > 0 ? p.mma_n1 : 16);
      const uint32_t idesc2 = idesc_bf16_f32(kBM, p.mma_n1 > 0 ? p.bn - p.mma_n1 : 16);
      const int stages = p.stages, bn = p.bn, mma_n = p.mma_n;
      const uint32_t full0 = smem_u32(full), empty0 = smem_u32(empty);
      const uint64_t desc_hi = sw128_kmajor_desc(0);
      const uint32_t a_lo0 = smem_u32(smem) >> 4, stage_lo = stage_bytes >> 4;
      const uint32_t sub_lo = (uint32_t)mma_n * 8u;   // mma_n rows of 128 B, in 16-byte units
      bool ok = true;
      int s = 0, ph = 0;
      for (int i = 0; i < nkb; ++i) {
        if (!mbar_wait(full0 + 8u * s, ph, abort_flag, p.spin)) {
          set_status(p.status, kStatusTimeoutMma);
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        mma_issued = true;
        const uint64_t da = desc_hi | (uint64_t)(a_lo0 + (uint32_t)s * stage_lo);
        const uint64_t db = da + (uint64_t)(kNA * (kATileBytes >> 4));
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          const uint64_t a_k = da + 2u * kk;            // +32 bytes along K
          uint64_t b_k = db + 2u * kk;
          if (PAIR) {   // one MMA per accumulator spans the whole token tile (mma_n == bn <= 256)
            tc_mma_f16_pair(tmem_base, a_k, b_k, idesc, acc);
            if (kNA == 2) tc_mma_f16_pair(tmem_base + bn, a_k + (kATileBytes >> 4), b_k, idesc, acc);
          } else if (p.mma_n1 > 0) {
            tc_mma_f16(tmem_base, a_k, b_k, idesc1, acc);
            tc_mma_f16(tmem_base + p.mma_n1, a_k, b_k + (uint64_t)(p.mma_n1 * 8), idesc2, acc);
          } else {
            for (int nb = 0; nb < bn; nb += mma_n, b_k += sub_lo) {
              tc_mma_f16(tmem_base + nb, a_k, b_k, idesc, acc);
              if (kNA == 2) tc_mma_f16(tmem_base + bn + nb, a_k + (kATileBytes >> 4), b_k, idesc, acc);
            }
          }
        }
        if (PAIR) {   // the stage is free in both CTAs
          tc_commit_pair(empty0 + 8u * s);
          tc_commit_pair(dsmem_addr(empty0 + 8u * s, 1));
        } else {
          tc_commit(empty0 + 8u * s);
        }
        if (++s == stages) { s = 0; ph ^= 1; }
      }
      if (ok) {
        if (PAIR) {
          tc_commit_pair(smem_u32(accb));
          tc_commit_pair(dsmem_addr(smem_u32(accb), 1));
        } else {
          tc_commit(smem_u32(accb));
        }
        mma_committed = true;
      }
    }
    __syncwarp();
  }

  // ---------------- epilogue: warps 2..9, two per TMEM lane quadrant (warp % 4); half h takes
  // the 16-column chunks h, h+2, h+4, ...
  const bool epi_warp = warp >= 2;
  const int q = warp & 3;
  const int half = (warp - 2) >> 2;
  const int row_local = q * 32 + lane;
  const int row = m0 + row_local;
  const bool row_ok = row < p.n_out;
  const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
  bool ok = true;
  bool copies_issued = false;   // split-K staging: this thread issued bulk copies into epib
  if (epi_warp) {
    pdl_wait();
    ok = mbar_wait(smem_u32(accb), 0, abort_flag, p.spin);
    if (!ok) {
      set_status(p.status, kStatusTimeoutEpilogue);
      *abort_flag = 1;
    }
    tc_fence_after();
  }

  if (p.splits == 1) {
    if (EPI == EESD_EPI_STORE || EPI == EESD_EPI_RESIDUAL || EPI == EESD_EPI_SWIGLU) {
      if (epi_warp && ok) {
        for (int c = half * 16; c < p.bn; c += 32) {
          float v[16], u[16];
          tmem_ld16(lane_base + c, v);
          if (EPI == EESD_EPI_SWIGLU) tmem_ld16(lane_base + p.bn + c, u);
          if (row_ok) epilogue_cols<EPI, 16>(p, n0 + c, row, v, u);
        }
      }
    } else {  // ARGMAX: logits rounded to bf16, max over this CTA's rows, then atomicMax
      unsigned long long* red = reinterpret_cast<unsigned long long*>(smem);  // stage memory is free now
      const int row2 = row + kBM;                      // two-tile head: this lane's row of the second tile
      const bool row2_ok = kNA == 2 && row2 < p.n_out;
      if (epi_warp && ok) {
        for (int c = half * 16; c < p.bn; c += 32) {
          float v[16], v2[16];
          tmem_ld16(lane_base + c, v);
          if (kNA == 2) tmem_ld16(lane_base + p.bn + c, v2);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            unsigned long long key = row_ok ? argmax_key(rnd<bf16>(v[j]), (uint32_t)row) : 0ull;
            if (kNA == 2 && row2_ok) {
              const unsigned long long k2 = argmax_key(rnd<bf16>(v2[j]), (uint32_t)row2);
              key = k2 > key ? k2 : key;
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
              const unsigned long long o = __shfl_xor_sync(0xffffffffu, key, off);
              key = o > key ? o : key;
            }
            if (lane == 0) red[(c + j) * 4 + q] = key;
          }
        }
      }
      if (epi_warp) epi_bar();
      if (epi_warp && ok) {
        for (int c = threadIdx.x - 64; c < p.bn; c += kEpiThreads) {
          const int t = n0 + c;
          if (t < p.n_tok) {
            unsigned long long k = red[c * 4];
            for (int w = 1; w < 4; ++w) k = red[c * 4 + w] > k ? red[c * 4 + w] : k;
            atomicMax(&p.keys[t], k);
          }
        }
      }
    }
  } else {
    // ---------------- split-K through L2.  CTA r of the cluster owns the token-column slice
    // [r * slice, (r + 1) * slice) of the tile.  Every CTA stores its fp32 partial of the columns
    // it does not own (laid out [column / 4][128 rows] float4: a warp's 32 rows are 512 contiguous
    // bytes), one cluster barrier (release / acquire at cluster scope) publishes them, then every
    // owner adds the splits in split order - its own straight from TMEM - and runs the epilogue.
    // The other splits' partials of the owned slice (one contiguous run per split) and, for the
    // residual epilogue, the slice's residual rows are brought into the idle stage memory by bulk
    // copies, so the owner phase waits for one round trip instead of one per 16-column chunk.
    // The cluster's CTAs are co-scheduled, so the barrier never waits on an unscheduled CTA.
    const int S = p.splits;
    const int rank = (int)cluster_rank();
    const int slice = ((p.bn + S - 1) / S + 15) / 16 * 16;
    const int own_lo = min(p.bn, rank * slice), own_hi = min(p.bn, own_lo + slice);
    const int own_w = own_hi - own_lo;                 // multiple of 16
    const size_t part_f4 = (size_t)p.acc_cols * 32;   // float4s in one split's partial tile
    float4* tile_parts = p.partials + (size_t)((out_tile * gridDim.x + tok_tile) * S) * part_f4;
    const uint32_t run_bytes = (uint32_t)own_w * 512u;              // one split, one accumulator
    const uint32_t part_stage = (uint32_t)(S - 1) * kNA * run_bytes;
    const int res_tokens = EPI == EESD_EPI_RESIDUAL && p.res_stage ? max(0, min(own_w, p.n_tok - (n0 + own_lo))) : 0;
    const uint32_t res_bytes = (uint32_t)res_tokens * 256u;
    const bool staged = own_w > 0 && part_stage + res_bytes <= (uint32_t)p.stages * stage_bytes;
    const uint32_t stage0 = smem_u32(smem);
    if (epi_warp && ok) {
      float4* mine = tile_parts + (size_t)rank * part_f4;
      for (int c = half * 16; c < p.bn; c += 32) {
        if (c >= own_lo && c < own_hi) continue;      // the owned slice stays in TMEM
#pragma unroll
        for (int part = 0; part < kNA; ++part) {
          float v[16];
          tmem_ld16(lane_base + part * p.bn + c, v);
          const int g0 = (part * p.bn + c) / 4;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            mine[(size_t)(g0 + j) * 128 + row_local] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
      }
      fence_proxy_async_global();   // the peers read these stores with bulk (async-proxy) copies
    }
    bool issuer_ok = true;
    if (staged && warp == 0 && lane == 0) {
      // the stage memory is free once every MMA has completed
      issuer_ok = mbar_wait(smem_u32(accb), 0, abort_flag, p.spin);
      if (issuer_ok) {
        copies_issued = true;
        mbar_arrive_expect_tx(smem_u32(epib), part_stage + res_bytes);
        for (int t = 0; t < res_tokens; ++t)
          bulk_g2s(stage0 + part_stage + (uint32_t)t * 256u, p.residual + (size_t)(n0 + own_lo + t) * p.ld_res + m0,
                   256u, smem_u32(epib));
      } else {
        set_status(p.status, kStatusTimeoutEpilogue);
        *abort_flag = 1;
      }
    }
    cluster_sync();
    if (staged && warp == 0 && lane == 0 && issuer_ok) {
      fence_proxy_async_global();
      uint32_t dst = stage0;
      for (int sp = 0; sp < S; ++sp) {
        if (sp == rank) continue;
        const float4* src = tile_parts + (size_t)sp * part_f4;
#pragma unroll
        for (int part = 0; part < kNA; ++part, dst += run_bytes)
          bulk_g2s(dst, src + (size_t)((part * p.bn + own_lo) / 4) * 128, run_bytes, smem_u32(epib));
      }
    }
    if (epi_warp && ok && staged) {
      if (!mbar_wait(smem_u32(epib), 0, abort_flag, p.spin)) {
        set_status(p.status, kStatusTimeoutEpilogue);
        *abort_flag = 1;
      } else {
        const float4* st4 = reinterpret_cast<const float4*>(smem);
        const bf16* res_s = reinterpret_cast<const bf16*>(smem + part_stage);
        for (int c = own_lo + half * 16; c < own_hi; c += 32) {
          float g[16], u[16];
#pragma unroll 1
          for (int sp = 0, k = 0; sp < S; ++sp) {
            float pg[16], pu[16];
            if (sp == rank) {
              tmem_ld16(lane_base + c, pg);
              if (kNA == 2) tmem_ld16(lane_base + p.bn + c, pu);
            } else {
              // staged run k of this split: [accumulator][own_w / 4][128] float4
              const float4* src = st4 + (size_t)k * kNA * (own_w / 4) * 128;
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float4 a = src[(size_t)((c - own_lo) / 4 + j) * 128 + row_local];
                pg[4 * j] = a.x;
                pg[4 * j + 1] = a.y;
                pg[4 * j + 2] = a.z;
                pg[4 * j + 3] = a.w;
                if (kNA == 2) {
                  const float4 b4 = src[(size_t)(own_w / 4 + (c - own_lo) / 4 + j) * 128 + row_local];
                  pu[4 * j] = b4.x;
                  pu[4 * j + 1] = b4.y;
                  pu[4 * j + 2] = b4.z;
                  pu[4 * j + 3] = b4.w;
                }
              }
              ++k;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              g[j] = sp == 0 ? pg[j] : g[j] + pg[j];
              if (kNA == 2) u[j] = sp == 0 ? pu[j] : u[j] + pu[j];
            }
          }
          if (row_ok) {
            float r[16];
            if (EPI == EESD_EPI_RESIDUAL) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int tl = c - own_lo + j;
                r[j] = tl < res_tokens ? __bfloat162float(res_s[tl * 128 + row_local]) : 0.f;
              }
              if (!p.res_stage) load_residual<EPI, 16>(p, n0 + c, row, r);
            }
            epilogue_cols_r<EPI, 16>(p, n0 + c, row, g, u, r);
          }
        }
      }
    } else if (epi_warp && ok) {
      for (int c = half * 16; c < p.bn; c += 32) {
        if (c < own_lo || c >= own_hi) continue;
        float g[16], u[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) g[j] = u[j] = 0.f;
#pragma unroll 2
        for (int sp = 0; sp < S; ++sp) {
          float pg[16], pu[16];
          if (sp == rank) {
            tmem_ld16(lane_base + c, pg);
            if (kNA == 2) tmem_ld16(lane_base + p.bn + c, pu);
          } else {
            const float4* src = tile_parts + (size_t)sp * part_f4;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float4 a = __ldcg(src + (size_t)(c / 4 + j) * 128 + row_local);
              pg[4 * j] = a.x;
              pg[4 * j + 1] = a.y;
              pg[4 * j + 2] = a.z;
              pg[4 * j + 3] = a.w;
              if (kNA == 2) {
                const float4 b4 = __ldcg(src + (size_t)((p.bn + c) / 4 + j) * 128 + row_local);
                pu[4 * j] = b4.x;
                pu[4 * j + 1] = b4.y;
                pu[4 * j + 2] = b4.z;
                pu[4 * j + 3] = b4.w;
              }
            }
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            g[j] = sp == 0 ? pg[j] : g[j] + pg[j];
            if (kNA == 2) u[j] = sp == 0 ? pu[j] : u[j] + pu[j];
          }
        }
        if (row_ok) epilogue_cols<EPI, 16>(p, n0 + c, row, g, u);
      }
    }
  }
  if (copies_issued && *abort_flag) {
    // the bulk copies this CTA issued land before it exits, even if its epilogue gave up
    mbar_drain(smem_u32(epib), 0);
  }
  tc_fence_before();
  __syncwarp();
  __syncthreads();
  // Every role has finished, so the abort flag is final.  After an abort, loads and MMAs may still
  // be in flight: the CTA leaves (and frees its TMEM) only once they have landed.  Each ring slot has
  // at most one load phase outstanding (the producer refills a slot only after its MMAs freed it), so
  // waiting for the phase of the last k-block loaded into each slot drains them all.  A CTA pair's
  // loads complete on the even CTA's barriers, which the even CTA drains before the closing cluster
  // barrier releases the odd one.
  if (*abort_flag) {
    if (warp == 0 && lane == 0 && (!PAIR || rank == 0)) {
      for (int slot = 0; slot < p.stages && slot < loads_issued; ++slot) {
        const int last = slot + (loads_issued - 1 - slot) / p.stages * p.stages;
        mbar_drain(smem_u32(&full[slot]), (uint32_t)(last / p.stages) & 1u);
      }
    }
    if (warp == 1 && lane == 0 && mma_issued) {
      if (mma_committed) {
        mbar_drain(smem_u32(accb), 0);
      } else {
        if (PAIR)
          tc_commit_pair(smem_u32(drainb));
        else
          tc_commit(smem_u32(drainb));
        mbar_drain(smem_u32(drainb), 0);
      }
    }
    tc_fence_before();
    __syncwarp();
    __syncthreads();
  }
  // a CTA of a pair leaves only when both are done: the even CTA's MMAs and commits reach the odd
  // CTA's TMEM and barriers, the odd CTA's loads reach the even CTA's barriers
  if (PAIR) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem_base, (uint32_t)p.tmem_cols);
    else
      tmem_dealloc(tmem_base, (uint32_t)p.tmem_cols);
  }
}

// ------------------------------------------------------------------ host side
PFN_encodeTiled_t g_encode = nullptr;
std::once_flag g_encode_once;
int g_mma_n_option = 0;   // 0: one MMA spans the whole token tile
int g_splits_option = 0;  // 0: split count from the weight shape
int g_stages_option = 0;  // 0: as many stages as the shared-memory budget holds
int g_pair_option = 1;    // 1: SwiGLU GEMMs whose row tiles pair up run on CTA pairs (cta_group::2)
int g_head_two_option = 1;  // 1: head launches of up to 256 tokens take two row tiles per CTA
// Token tiles above 256 on one CTA take two MMAs per k-step.  Equal halves (e.g. 160 + 160 at 320
// tokens) measured slower than 192 + 128 (or 256 + 64): 250.4 -> 235.5 us per 320-token layer,
// bit-identical.  0 restores equal halves.
int g_split_n_option = 192;

int next_pow2(int v) {
  int p = 32;
  while (p < v) p <<= 1;
  return p;
}

template <int EPI, bool PAIR>
int ensure_smem_attr(size_t bytes) {
  static size_t set = 0;
  if (bytes > set) {
    if (cudaFuncSetAttribute(tc_gemm_kernel<EPI, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) !=
        cudaSuccess)
      return EESD_ERR_CUDA;
    set = bytes;
  }
  return EESD_OK;
}

template <int EPI>
int launch(const TcPlan& pl, const CUtensorMap& map_w, const CUtensorMap& map_x, const TcParams& p,
           cudaStream_t stream) {
  if constexpr (EPI == EESD_EPI_SWIGLU) {
    if (pl.pair) {   // CTA pairs: grid (pair member, token tile, 256-row tile), clusters of 2
      int rc = ensure_smem_attr<EPI, true>(pl.smem);
      if (rc) return rc;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2, pl.tok_tiles, pl.out_tiles / 2);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = pl.smem;
      cfg.stream = stream;
      cudaLaunchAttribute attr[2];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[1].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 2;
      return cudaLaunchKernelEx(&cfg, tc_gemm_kernel<EPI, true>, map_w, map_x, p) == cudaSuccess ? EESD_OK
                                                                                               : EESD_ERR_CUDA;
    }
  }
  int rc = ensure_smem_attr<EPI, false>(pl.smem);
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.tok_tiles, EPI == EESD_EPI_ARGMAX2_INTERNAL ? (pl.out_tiles + 1) / 2 : pl.out_tiles, pl.splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = pl.splits;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, tc_gemm_kernel<EPI, false>, map_w, map_x, p) == cudaSuccess ? EESD_OK : EESD_ERR_CUDA;
}

}  // namespace

PFN_encodeTiled_t tensor_map_encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_encodeTiled_t>(fn);
  });
  return g_encode;
}

int encode_kmajor_map(CUtensorMap* map, const void* base, int rows, int k, int box_rows) {
  PFN_encodeTiled_t enc = tensor_map_encoder();
  if (!enc) return EESD_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (k % 8) || box_rows < 1 || box_rows > 256) return EESD_ERR_ARG;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)k * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? EESD_OK : EESD_ERR_CUDA;
}

int encode_packed_map(CUtensorMap* map, const void* base, int rows, int k) {
  PFN_encodeTiled_t enc = tensor_map_encoder();
  if (!enc) return EESD_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (k % kBK) || rows <= 0) return EESD_ERR_ARG;
  const cuuint64_t tiles = (cuuint64_t)((rows + kBM - 1) / kBM) * (k / kBK);
  cuuint64_t dims[3] = {(cuuint64_t)kBK, (cuuint64_t)kBM, tiles};
  cuuint64_t strides[2] = {(cuuint64_t)kBK * 2, (cuuint64_t)kATileBytes};
  cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)kBM, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? EESD_OK : EESD_ERR_CUDA;
}

size_t packed_weight_bytes(int rows, int k) {
  return (size_t)((rows + kBM - 1) / kBM) * (size_t)((k + kBK - 1) / kBK) * kATileBytes;
}

namespace {
// out[(tile * 128 + r) * 64 + c] = w[(mt * 128 + r) * k + kb * 64 + c], tile = mt * KB + kb; rows past
// the end are zero.  One thread per 16-byte chunk: writes are contiguous, reads stride by row.
__global__ void pack_weight_kernel(const uint4* __restrict__ w, uint4* __restrict__ out, int rows, int k, size_t n) {
  const size_t o = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= n) return;
  const int kb_total = k / kBK;
  const size_t tile = o >> 10;                 // 128 rows x 8 chunks per tile
  const int r = (int)((o >> 3) & 127), c = (int)(o & 7);
  const int mt = (int)(tile / kb_total), kb = (int)(tile % kb_total);
  const int row = mt * kBM + r;
  out[o] = row < rows ? w[((size_t)row * k + kb * kBK) / 8 + c] : make_uint4(0, 0, 0, 0);
}
}  // namespace

int pack_weight(const void* w, int rows, int k, void* out, cudaStream_t s) {
  if (!w || !out || rows <= 0 || k <= 0 || k % kBK) return EESD_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(out)) & 15) return EESD_ERR_ARG;
  const size_t n = packed_weight_bytes(rows, k) / 16;
  pack_weight_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(static_cast<const uint4*>(w), static_cast<uint4*>(out),
                                                                 rows, k, n);
  return cudaPeekAtLastError() == cudaSuccess ? EESD_OK : EESD_ERR_CUDA;
}

void tc_set_mma_n(int n) { g_mma_n_option = n; }
void tc_set_splits(int n) { g_splits_option = n; }
void tc_set_stages(int n) { g_stages_option = n; }
void tc_set_pair(int n) { g_pair_option = n; }
void tc_set_head_two_tiles(int n) { g_head_two_option = n; }
void tc_set_split_n(int n) { g_split_n_option = n; }

TcPlan tc_plan(int n_tok, int n_out, int k, int epi) {
  TcPlan pl{};
  const int mma_fixed = g_mma_n_option;
  const int max_tile = epi == EESD_EPI_SWIGLU ? 256 : 384;
  pl.tok_tiles = (n_tok + max_tile - 1) / max_tile;
  const int per = (n_tok + pl.tok_tiles - 1) / pl.tok_tiles;
  if (mma_fixed > 0) {
    pl.mma_n = mma_fixed;
    pl.bn = (per + mma_fixed - 1) / mma_fixed * mma_fixed;
    if (pl.bn > max_tile) pl.bn = max_tile / mma_fixed * mma_fixed;
    if (pl.bn > 256 && (pl.bn / 2) % 16) pl.bn = 256 / mma_fixed * mma_fixed;
    pl.tok_tiles = (n_tok + pl.bn - 1) / pl.bn;
  } else if (per <= 256) {
    pl.bn = std::max(16, (per + 15) / 16 * 16);
    pl.mma_n = pl.bn;
  } else {
    pl.bn = (per + 31) / 32 * 32;
    pl.mma_n = pl.bn / 2;
  }
  pl.b_boxes = pl.bn > 256 ? 2 : 1;
  pl.out_tiles = (n_out + kBM - 1) / kBM;
  pl.kb_total = (k + kBK - 1) / kBK;
  // split count from the weight shape only (never from n_tok): weights with fewer than ~100 row
  // tiles are split so that about one wave of 148 SMs streams them, using 2 or 4 splits (clusters of
  // 2 or 4 CTAs pack into every GPC; 3 leaves clusters waiting for a second wave), with at least 8
  // k-blocks (512 of K) per split
  int s = 1;
  if (epi != EESD_EPI_ARGMAX_INTERNAL && pl.out_tiles < 100) {
    const int cap = std::min(148 / std::max(pl.out_tiles, 1), std::min(pl.kb_total / 8, 4));
    s = cap >= 4 ? 4 : (cap >= 2 ? 2 : 1);
  }
  if (g_splits_option > 0 && epi != EESD_EPI_ARGMAX_INTERNAL) s = std::min(g_splits_option, kMaxSplits);
  pl.kb_per = (pl.kb_total + s - 1) / s;
  pl.splits = (pl.kb_total + pl.kb_per - 1) / pl.kb_per;
  // The head (no split) takes two 128-row tiles per CTA where both accumulators fit in TMEM: each
  // stage then carries 32 KB of weights per barrier round trip instead of 16 KB.  Every logit is
  // the same k-ordered sum either way and the argmax is order-free, so the choice may depend on
  // n_tok.
  pl.argmax2 = epi == EESD_EPI_ARGMAX_INTERNAL && g_head_two_option && pl.bn <= 256;
  const int na = (epi == EESD_EPI_SWIGLU || pl.argmax2) ? 2 : 1;
  // CTA pairs for unsplit SwiGLU tiles (a whole number of 256-row tiles, one MMA per accumulator);
  // the choice depends on the weight shape and the option only, never on n_tok
  pl.pair = epi == EESD_EPI_SWIGLU && g_pair_option && mma_fixed == 0 && pl.splits == 1 && n_out % (2 * kBM) == 0 &&
            pl.bn <= 256;
  if (pl.pair) pl.mma_n = pl.bn;
  const size_t stage = (size_t)na * kATileBytes + (size_t)(pl.pair ? pl.bn / 2 : pl.bn) * kBK * 2;
  pl.stages = (int)std::min<size_t>(8, kSmemBudget / stage);
  if (g_stages_option >= 2 && (size_t)g_stages_option * stage <= kSmemBudget) pl.stages = g_stages_option;
  pl.smem = (size_t)pl.stages * stage + 1024 + 256;
  pl.acc_cols = na * pl.bn;
  pl.tmem_cols = next_pow2(pl.acc_cols);
  // split-K partial tiles: one fp32 tile per (output tile, token tile, split)
  pl.partial_bytes = pl.splits > 1 ? (size_t)pl.out_tiles * pl.tok_tiles * pl.splits * 128 * (size_t)pl.acc_cols * 4 : 0;
  return pl;
}

size_t tc_partial_bytes_max(int max_tok, int n_out, int k, int epi) {
  size_t b = 0;
  for (int n = 1; n <= max_tok; ++n) b = std::max(b, tc_plan(n, n_out, k, epi).partial_bytes);
  return b;
}

int tc_gemm_launch(int epi, const CUtensorMap& map_w, const void* x, int n_tok, int n_out, int k, int up_offset,
                   const void* residual, int ld_res, void* y, int ld_y, unsigned long long* keys, int* status,
                   cudaStream_t stream, int a_packed, const TcScratch& scratch) {
  if (a_packed && (k % kBK || up_offset % kBM)) return EESD_ERR_ARG;
  if (n_tok <= 0 || n_out <= 0 || k <= 0) return EESD_ERR_ARG;
  const TcPlan pl = tc_plan(n_tok, n_out, k, epi);
  if (pl.stages < 2) return EESD_ERR_ARG;
  if (pl.partial_bytes && (!scratch.partials || scratch.partial_bytes < pl.partial_bytes ||
                           (reinterpret_cast<uintptr_t>(scratch.partials) & 15)))
    return EESD_ERR_ARG;
  CUtensorMap map_x;
  int rc = encode_kmajor_map(&map_x, x, n_tok, k, (pl.b_boxes == 2 || pl.pair) ? pl.bn / 2 : pl.bn);
  if (rc) return rc;
  TcParams p{};
  p.n_tok = n_tok;
  p.n_out = n_out;
  p.K = k;
  p.bn = pl.bn;
  p.b_boxes = pl.b_boxes;
  p.mma_n = pl.mma_n;
  p.kb_total = pl.kb_total;
  p.kb_per = pl.kb_per;
  p.splits = pl.splits;
  p.stages = pl.stages;
  p.up_offset = pl.argmax2 ? kBM : up_offset;   // two-tile head: the second A tile is the next 128 rows
  p.tmem_cols = pl.tmem_cols;
  p.a_packed = a_packed;
  p.acc_cols = pl.acc_cols;
  {
    const int n1 = g_split_n_option, n2 = pl.bn - n1;
    const bool kna1 = !(epi == EESD_EPI_SWIGLU || pl.argmax2);
    p.mma_n1 = (n1 > 0 && kna1 && !pl.pair && pl.bn > 256 && pl.mma_n * 2 == pl.bn && n1 % 16 == 0 && n2 % 16 == 0 &&
                n1 <= 256 && n2 >= 16 && n2 <= 256)
                   ? n1
                   : 0;
  }
  // residual rows of an owned slice by 256-byte bulk copies: whole 128-row tiles, 16-byte aligned rows
  p.res_stage = epi == EESD_EPI_RESIDUAL && n_out % kBM == 0 && ld_res % 8 == 0 &&
                (reinterpret_cast<uintptr_t>(residual) & 15) == 0;
  p.partials = static_cast<float4*>(scratch.partials);
  p.residual = static_cast<const bf16*>(residual);
  p.ld_res = ld_res;
  p.y = static_cast<bf16*>(y);
  p.ld_y = ld_y;
  p.keys = keys;
  p.status = status;
  p.spin = spin_limit();
  switch (epi) {
    case EESD_EPI_STORE: return launch<EESD_EPI_STORE>(pl, map_w, map_x, p, stream);
    case EESD_EPI_RESIDUAL: return launch<EESD_EPI_RESIDUAL>(pl, map_w, map_x, p, stream);
    case EESD_EPI_SWIGLU: return launch<EESD_EPI_SWIGLU>(pl, map_w, map_x, p, stream);
    case EESD_EPI_ARGMAX_INTERNAL:
      return pl.argmax2 ? launch<EESD_EPI_ARGMAX2_INTERNAL>(pl, map_w, map_x, p, stream)
                        : launch<EESD_EPI_ARGMAX_INTERNAL>(pl, map_w, map_x, p, stream);
    default: return EESD_ERR_ARG;
  }
}

}  // namespace eesd
