// prefill_full on B200: a whole prompt of C tokens (C = bucket width, a multiple of
// 128) through the 32 layers in one pass, emitting its K/V cache.
//
// Replaces the reference's KV-free prefill graph (PrefillLayer.forward,
// src/rngd_pd/kernels/prefill_full.py:56-76, driven by FullPrefillEngine,
// src/rngd_pd/engines/prefill_full.py:337-388).  Per layer:
//   QKV GEMM (+ RoPE, K/V emission)  -> causal attention within the prompt
//   -> O GEMM (+ residual)           -> gate/up GEMM (+ SwiGLU) -> down GEMM (+ residual)
//
// GEMMs run on tcgen05 (pfgemm_kernel): D[n][t] = sum_k W[n][k] * h[t][k] with a
// 128-row weight tile as A and a tile of NT tokens as B.  The fp32 activations
// enter as two bf16 operand rows per token, hi = bf16(h) and lo = bf16(h - hi),
// issued as two MMAs into the same TMEM accumulator (D = W*hi + W*lo), which keeps
// fp32-level accuracy.  Scheduling is persistent stream-K over (weight tile,
// token tile, K block), as for decode (decode_tc.cu): one CTA per SM, equal work,
// deterministic in-order reduction of tiles cut between CTAs.  A unit cut between CTAs is
// summed by its first owner (its own piece stays in TMEM): the other owners store their
// pieces and publish each with one release flag = (shape tag, unit epoch + 1), the first
// owner acquires the flags (bounded wait), adds the pieces in K order and advances the epoch.
//
// Operand layout: act [2C][K] bf16, rows 0..C-1 = hi of token t, rows C..2C-1 =
// lo.  RMSNorm is folded exactly as in decode: the producer of x writes x * w and
// per-128-column sums of squares ss[H/128][C]; the consumer scales token t's row
// by 1/sqrt(sum/H + eps).
//
// KV output ("prefill layout"): bf16 [L][2][NKV][S][HD], K then V per layer, a
// position's 128 values contiguous; positions >= P (prompt length) stay as the
// caller zeroed them (engines/prefill_full.py:319-335 pads with zeros).
#include "tc.cuh"

namespace rngd {

__device__ int g_status_prefill = 0;

constexpr int PBM = 128, PBK = 64;
constexpr int P_GROUPS = 4;    // epilogue warpgroups, each a quarter of every 32-token chunk
constexpr int P_EPI = 128 * P_GROUPS;  // epilogue threads
constexpr int P_HALF = 32 / P_GROUPS;  // tokens of a chunk per warpgroup
constexpr int P_YS_LD = P_HALF + 1;    // smem pitch (odd) of a warpgroup's [128][P_HALF] exchange buffer
constexpr int P_MAXPIECE = 2;  // split-unit pieces whose loads are issued together (4 spills at
                               // the 96-register cap of the four-warpgroup epilogue and ran slower)

// MT weight tiles (128 rows each) share every token tile: with MT = 2 a 64 KB stage
// carries 32 KB of weights and 32 KB of activations (hi + lo) for twice the MMA work of
// MT = 1, halving the activation traffic per FLOP.
template <int NT, int MT>
struct PCfg {
  static constexpr int A_BYTES = MT * PBM * PBK * 2;  // MT x 16 KB of weight rows
  static constexpr int B_BYTES = NT * PBK * 2;        // one token tile (hi or lo)
  static constexpr int STAGE = A_BYTES + 2 * B_BYTES;
  static constexpr int STAGES = MT == 2 ? 3 : 4;
  static constexpr int TMEM_COLS = 2 * MT * NT;       // MT accumulators, double-buffered
  static constexpr size_t BAR_BYTES = (2 * STAGES + 5) * 8;
  // ring | barriers | tmem slot, flag | s_scale [NT] | ys [P_GROUPS][128][P_YS_LD] | s_red [P_GROUPS][4][P_HALF]
  static constexpr size_t SMEM = 1024 + STAGES * STAGE + BAR_BYTES + 64 + NT * 4 +
                                 P_GROUPS * PBM * P_YS_LD * 4 + P_GROUPS * 4 * P_HALF * 4;
};

enum PEpi : int { PEPI_QKV = 0, PEPI_RESID = 1, PEPI_SWIGLU = 2 };

struct PArgs {
  int N, K, nkb, ntok, total, maxseg, layer;
  int C, P;
  float* partial;  // [units][maxseg][MT][NT][128] pieces of split units (slot 0's never stored)
  int* counters;   // [units] split epochs, then [units][maxseg] piece flags; zeroed once
  int nunits, tag;  // units of this launch; 1..15, distinct for GEMM shapes sharing the scratch
  int lo;           // 1: W*hi + W*lo (fp32-level operand); 0: W*hi only (one bf16 operand row)
  const float* ss_in;  // [ss_tiles][C]
  int ss_tiles;
  float eps, inv_h;
  // QKV
  const float* inv;
  float* q;
  int ldq;
  uint16_t* kv;  // this layer's [2][NKV][S][HD]
  uint16_t* vt;  // V^T scratch [NKV][HD][C] for the attention (the act2 buffer, idle until the MLP)
  int NH, NKV, S;
  // RESID
  float* x;
  int ldx;
  const float* w_next;
  uint16_t* act_next;
  int ld_next;
  float* ss_out;
  // SWIGLU
  uint16_t* act_out;
  int ld_act;
  // per-CTA timeline [grid][16] (diagnostics; only a library built with RNGD_TRACE=1 records it)
  unsigned long long* trace;
};

// named barriers: 1 + g = epilogue warpgroup g (128 threads), 1 + P_GROUPS = all of them
__device__ __forceinline__ void pf_sync_g(int g) { asm volatile("bar.sync %0, 128;" ::"r"(1 + g) : "memory"); }
__device__ __forceinline__ void pf_sync_all() {
  asm volatile("bar.sync %0, %1;" ::"n"(1 + P_GROUPS), "n"(P_EPI) : "memory");
}
// this thread's P_HALF accumulator columns from TMEM
__device__ __forceinline__ void pf_tmem_ld(uint32_t taddr, float* v) {
  if constexpr (P_HALF == 16)
    tmem_ld_32x32b_x16(taddr, v);
  else
    tmem_ld_32x32b_x8(taddr, v);
}
__device__ __forceinline__ void pf_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <int EPI, int NT, int MT>
__global__ void __launch_bounds__(64 + P_EPI, 1) pfgemm_kernel(const __grid_constant__ CUtensorMap tmW,
                                                              const __grid_constant__ CUtensorMap tmX, PArgs a) {
  using Cfg = PCfg<NT, MT>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(base + STAGES * Cfg::STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint64_t* epi_done = acc_empty + 2;   // the epilogue threads are past their last TMEM read
  uint32_t* tmem_slot = (uint32_t*)((uint8_t*)full + Cfg::BAR_BYTES);
  float* s_scale = (float*)((uint8_t*)full + Cfg::BAR_BYTES + 64);   // [NT] RMS scale of the unit's tokens
  float* ys_all = s_scale + NT;                                      // [P_GROUPS][128][P_YS_LD]
  float* s_red_all = ys_all + P_GROUPS * PBM * P_YS_LD;              // [P_GROUPS][4][P_HALF]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  const long f0 = (long)cta * a.total / G, f1 = (long)(cta + 1) * a.total / G;
  // unit u = (weight-tile group u % ngrp, token tile u / ngrp): the token tiles of one group
  // are far apart in u, so different CTAs stream the same weights at about the same time
  // and the second read hits L2 instead of HBM
  const int ngrp = a.N / (MT * PBM);
  const bool use_lo = a.lo != 0;
  // RNGD_TRACE == 0 (the product build): tr is a constant null and every stamp below folds away.
  // Slots: 0 start, 1 TMA past the dependency wait, 2 first full stage, 3 last MMA commit,
  // 4 / 5 / 6 last unit: accumulator ready / pieces acquired / epilogue done, 7 first accumulator
  // ready, 8 last unit's owners, 9 this CTA's slot in it, 10 epilogue past the dependency wait
  unsigned long long* tr = (RNGD_TRACE && a.trace != nullptr) ? a.trace + (size_t)cta * 16 : nullptr;
  if (tr != nullptr && threadIdx.x == 0) tr[0] = globaltimer();
  const uint32_t stage_tx = (uint32_t)(Cfg::A_BYTES + (use_lo ? 2 : 1) * Cfg::B_BYTES);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], P_EPI);
    }
    mbar_init(epi_done, P_EPI);
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const long nk = f1 - f0;
      const long pre = nk < STAGES ? nk : STAGES;
      for (long i = 0; i < pre; i++) {
        const long f = f0 + i;
        const long u = f / a.nkb;
        const int kb = (int)(f - u * a.nkb), mg = (int)(u % ngrp);
        uint8_t* st = base + i * Cfg::STAGE;
        mbar_arrive_expect_tx(&full[i], stage_tx);
        tma_load_3d(st, &tmW, &full[i], kb * PBK, mg * MT * PBM, a.layer);
      }
      grid_dep_wait();
      if (tr != nullptr) tr[1] = globaltimer();
      for (long i = 0; i < pre; i++) {
        const long f = f0 + i;
        const long u = f / a.nkb;
        const int kb = (int)(f - u * a.nkb), jt = (int)(u / ngrp);
        uint8_t* st = base + i * Cfg::STAGE;
        tma_load_2d(st + Cfg::A_BYTES, &tmX, &full[i], kb * PBK, jt * NT);
        if (use_lo) tma_load_2d(st + Cfg::A_BYTES + Cfg::B_BYTES, &tmX, &full[i], kb * PBK, a.C + jt * NT);
      }
      for (long i = pre; i < nk; i++) {
        const int s = (int)(i % STAGES);
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, ST_TMA_WAIT, &g_status_prefill)) break;
        const long f = f0 + i;
        const long u = f / a.nkb;
        const int kb = (int)(f - u * a.nkb), mg = (int)(u % ngrp), jt = (int)(u / ngrp);
        uint8_t* st = base + s * Cfg::STAGE;
        mbar_arrive_expect_tx(&full[s], stage_tx);
        tma_load_3d(st, &tmW, &full[s], kb * PBK, mg * MT * PBM, a.layer);
        tma_load_2d(st + Cfg::A_BYTES, &tmX, &full[s], kb * PBK, jt * NT);
        if (use_lo) tma_load_2d(st + Cfg::A_BYTES + Cfg::B_BYTES, &tmX, &full[s], kb * PBK, a.C + jt * NT);
      }
      grid_dep_launch();
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(PBM, NT);
      long i = 0;
      int seg = 0;
      bool ok = true;
      for (long f = f0; f < f1 && ok; seg++) {
        const long u = f / a.nkb;
        const long fend = (u + 1) * a.nkb < f1 ? (u + 1) * a.nkb : f1;
        const int buf = seg & 1;
        ok = mbar_wait(&acc_empty[buf], ((uint32_t)(seg >> 1) & 1u) ^ 1u, ST_MMA_WAIT, &g_status_prefill);
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * MT * NT);
        for (long g = f; g < fend && ok; g++, i++) {
          const int s = (int)(i % STAGES);
          const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
          ok = mbar_wait(&full[s], ph, ST_MMA_WAIT, &g_status_prefill);
          if (!ok) break;
          if (tr != nullptr && i == 0) tr[2] = globaltimer();
          tc_fence_after();
          const uint32_t sa = smem_u32(base + s * Cfg::STAGE);
          const uint32_t sh = sa + Cfg::A_BYTES, sl = sh + Cfg::B_BYTES;
#pragma unroll
          for (int kk = 0; kk < PBK / 16; kk++) {
            const uint64_t hd = sw128_kmajor_desc(sh + kk * 32), ld_ = sw128_kmajor_desc(sl + kk * 32);
#pragma unroll
            for (int tt = 0; tt < MT; tt++) {  // tile tt: weight rows 128*tt.. of the stage, accumulator tt
              const uint64_t ad = sw128_kmajor_desc(sa + tt * PBM * 128 + kk * 32);
              const uint32_t dt = d + (uint32_t)(tt * NT);
              umma_bf16(dt, ad, hd, idesc, (g != f || kk != 0) ? 1u : 0u);
              if (use_lo) umma_bf16(dt, ad, ld_, idesc, 1u);
            }
          }
          umma_commit(&empty[s]);
        }
        umma_commit(&acc_full[buf]);
        f = fend;
      }
      if (tr != nullptr) tr[3] = globaltimer();
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps 2..: P_GROUPS warpgroups over the same 128 TMEM lanes.
    // Thread (group g, row r) owns row r of the tile for tokens P_HALF*g .. P_HALF*g + P_HALF-1 of
    // every 32-token chunk.  The last unit's epilogue is on the critical path of the pass (the
    // next GEMM reads every column it writes), and it shortens with more warps sharing it: with
    // two warpgroups instead of one it took 0.56-0.70x as long.
    grid_dep_wait();
    const int r = ((warp & 3) << 5) | lane;
    const int et = threadIdx.x - 64;   // 0 .. P_EPI-1
    if (tr != nullptr && et == 0) tr[10] = globaltimer();
    const int g = et >> 7;             // warpgroup
    const int eg = et & 127;           // index within the warpgroup
    float* ys = ys_all + g * PBM * P_YS_LD;
    float* s_red = s_red_all + g * 4 * P_HALF;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    int seg = 0;
    for (long f = f0; f < f1; seg++) {
      const long u = f / a.nkb;
      const long ustart = u * a.nkb;
      const long fend = ustart + a.nkb < f1 ? ustart + a.nkb : f1;
      const int mg = (int)(u % ngrp), jt = (int)(u / ngrp);
      const int buf = seg & 1;
      // epoch of the unit's split, read before the accumulator wait (only the unit's first owner
      // advances it, after every piece of this launch was published under the value read here)
      const int epoch = a.maxseg > 1 ? __ldcg(a.counters + u) : 0;
      // RMS scales of this unit's NT tokens, read while the accumulator is still being built:
      // token jt*NT + i's sum over the ss tiles in tile order, loads batched 16 at a time
      if (EPI != PEPI_RESID && a.ss_in != nullptr) {
        pf_sync_all();  // every warpgroup is past the previous unit's scales
        for (int i = et; i < NT; i += P_EPI) {
          const int tok = jt * NT + i;
          float ssum = 0.f;
          for (int t0 = 0; t0 < a.ss_tiles; t0 += 16) {
            float v16[16];
#pragma unroll
            for (int j = 0; j < 16; j++) v16[j] = t0 + j < a.ss_tiles ? a.ss_in[(size_t)(t0 + j) * a.C + tok] : 0.f;
#pragma unroll
            for (int j = 0; j < 16; j++)
              if (t0 + j < a.ss_tiles) ssum += v16[j];
          }
          s_scale[i] = 1.0f / sqrtf(ssum * a.inv_h + a.eps);
        }
        pf_sync_all();
      }
      mbar_wait(&acc_full[buf], (uint32_t)(seg >> 1) & 1u, ST_EPI_WAIT, &g_status_prefill);
      __syncwarp();
      tc_fence_after();
      const int first = owner_of(ustart, a.total, G), last = owner_of(ustart + a.nkb - 1, a.total, G);
      const int nseg = last - first + 1;
      const bool tlast = tr != nullptr && et == 0 && fend == f1;
      if (tr != nullptr && et == 0 && seg == 0) tr[7] = globaltimer();
      if (tlast) {
        tr[4] = globaltimer();
        tr[8] = (unsigned long long)nseg;
        tr[9] = (unsigned long long)(cta - first);
      }
      const uint32_t tbase0 = tmem + lane_base + (uint32_t)(buf * MT * NT);
      bool run = true;
      const int slot = cta - first;
      const uint32_t flag = ((uint32_t)a.tag << 28) | ((uint32_t)(epoch + 1) & 0x0FFFFFFFu);
      int* pflags = a.counters + a.nunits + (size_t)u * a.maxseg;
      if (nseg > 1 && slot > 0) {
        // a later piece of the unit: store it, publish it with one release, no wait
        for (int tt = 0; tt < MT; tt++) {
          float* pdst = a.partial + (((size_t)u * a.maxseg + slot) * MT + tt) * NT * PBM;
          for (int cc = 0; cc < NT / 32; cc++) {
            float v[P_HALF];
            pf_tmem_ld(tbase0 + tt * NT + cc * 32 + g * P_HALF, v);
#pragma unroll
            for (int i = 0; i < P_HALF; i++) __stcg(pdst + (size_t)(cc * 32 + g * P_HALF + i) * PBM + r, v[i]);
          }
        }
        tc_fence_before();
        pf_arrive(&acc_empty[buf]);
        pf_sync_all();  // every thread's piece stores precede the release below
        if (et == 0) asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(pflags + slot), "r"(flag) : "memory");
        if (tlast) tr[5] = tr[6] = globaltimer();
        run = false;
      } else if (nseg > 1) {
        // the unit's first piece is this CTA's own (in TMEM): wait (bounded) for the others'
        // flags; the barrier then orders every thread's piece loads after the acquires
        if (et == 0) {
          uint64_t t0 = 0;
          for (int sl = 1; sl < nseg; sl++) {
            while (true) {
              uint32_t v;
              asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(pflags + sl) : "memory");
              if (v == flag) break;
              const uint64_t now = globaltimer();
              if (t0 == 0) {
                t0 = now;
              } else if (now - t0 > kWaitTimeoutNs) {
                atomicCAS(&g_status_prefill, 0, ST_PIECE_WAIT);
                break;
              }
            }
          }
        }
        pf_sync_all();
      }
      if (tlast && run) tr[5] = globaltimer();
      if (run) {
       for (int tt = 0; tt < MT; tt++) {
        const int mt = mg * MT + tt;  // weight tile of this accumulator
        const int n = mt * PBM + r;
        for (int cc = 0; cc < NT / 32; cc++) {
          const int t0 = jt * NT + cc * 32 + g * P_HALF;  // first token of this thread's half chunk
          float xo[P_HALF];  // RESID: the residual row, loaded with the pieces (one round trip)
          if constexpr (EPI == PEPI_RESID) {
#pragma unroll
            for (int i = 0; i < P_HALF; i++) xo[i] = a.x[(size_t)(t0 + i) * a.ldx + n];
          }
          float y[P_HALF];
          pf_tmem_ld(tbase0 + tt * NT + cc * 32 + g * P_HALF, y);  // piece 0: this CTA's own
          if (nseg > 1) {
            for (int s0 = 1; s0 < nseg; s0 += P_MAXPIECE) {  // later pieces added in K order
              float pv[P_MAXPIECE][P_HALF];
#pragma unroll
              for (int q = 0; q < P_MAXPIECE; q++) {
                if (s0 + q < nseg) {
                  const float* src = a.partial + (((size_t)u * a.maxseg + s0 + q) * MT + tt) * NT * PBM +
                                     (size_t)(cc * 32 + g * P_HALF) * PBM + r;
#pragma unroll
                  for (int i = 0; i < P_HALF; i++) pv[q][i] = __ldcg(src + (size_t)i * PBM);
                }
              }
#pragma unroll
              for (int q = 0; q < P_MAXPIECE; q++) {
                if (s0 + q < nseg) {
#pragma unroll
                  for (int i = 0; i < P_HALF; i++) y[i] += pv[q][i];
                }
              }
            }
          }
          if (EPI != PEPI_RESID && a.ss_in != nullptr) {
#pragma unroll
            for (int i = 0; i < P_HALF; i++) y[i] *= s_scale[cc * 32 + g * P_HALF + i];
          }
          if constexpr (EPI == PEPI_RESID) {
#pragma unroll
            for (int i = 0; i < P_HALF; i++) {
              const float xn = xo[i] + y[i];
              a.x[(size_t)(t0 + i) * a.ldx + n] = xn;
              y[i] = xn;
            }
            if (a.act_next != nullptr) {
              const float w = a.w_next[n];
#pragma unroll
              for (int i = 0; i < P_HALF; i++) {
                const float h = y[i] * w;
                const uint16_t hi = f2bf_bits(h);
                a.act_next[(size_t)(t0 + i) * a.ld_next + n] = hi;
                a.act_next[(size_t)(a.C + t0 + i) * a.ld_next + n] = f2bf_bits(h - bf2f(hi));
              }
#pragma unroll
              for (int i = 0; i < P_HALF; i++) {
                const float sq = warp_sum(y[i] * y[i]);
                if (lane == 0) s_red[(warp & 3) * P_HALF + i] = sq;
              }
              pf_sync_g(g);
              if (eg < P_HALF)
                a.ss_out[(size_t)mt * a.C + t0 + eg] =
                    (s_red[eg] + s_red[P_HALF + eg]) + (s_red[2 * P_HALF + eg] + s_red[3 * P_HALF + eg]);
            }
          } else if constexpr (EPI == PEPI_QKV) {
#pragma unroll
            for (int i = 0; i < P_HALF; i++) ys[r * P_YS_LD + i] = y[i];
            pf_sync_g(g);
            const int head = mt;
            const int idx = r & 63;
            const bool lo_half = r < 64;
            const int partner = r ^ 64;
            if (head < a.NH + a.NKV) {
              const float invf = a.inv[idx];
#pragma unroll 8
              for (int i = 0; i < P_HALF; i++) {
                const int t = t0 + i;
                float sn, cs;
                sincosf((float)t * invf, &sn, &cs);
                const float other = ys[partner * P_YS_LD + i];
                const float o = lo_half ? y[i] * cs - other * sn : y[i] * cs + other * sn;
                if (head < a.NH) {  // q as the attention's hi/lo bf16 operand [2][C][NH*HD]
                  uint16_t* qb = reinterpret_cast<uint16_t*>(a.q);
                  const uint16_t hi = f2bf_bits(o);
                  qb[(size_t)t * a.ldq + n] = hi;
                  qb[(size_t)(a.C + t) * a.ldq + n] = f2bf_bits(o - bf2f(hi));
                } else if (t < a.P) {
                  a.kv[(((size_t)(head - a.NH)) * a.S + t) * 128 + r] = f2bf_bits(o);
                }
              }
            } else {
              const int vh = head - a.NH - a.NKV;
              uint32_t packed[P_HALF / 2];  // this dimension's P_HALF tokens for V^T (zero past the prompt)
#pragma unroll
              for (int i = 0; i < P_HALF; i += 2) {
                const int t = t0 + i;
                const uint16_t v0 = t < a.P ? f2bf_bits(y[i]) : 0, v1 = t + 1 < a.P ? f2bf_bits(y[i + 1]) : 0;
                packed[i / 2] = (uint32_t)v0 | ((uint32_t)v1 << 16);
                if (t < a.P) a.kv[(((size_t)(a.NKV + vh)) * a.S + t) * 128 + r] = v0;
                if (t + 1 < a.P) a.kv[(((size_t)(a.NKV + vh)) * a.S + t + 1) * 128 + r] = v1;
              }
              uint4* vrow = reinterpret_cast<uint4*>(a.vt + ((size_t)vh * 128 + r) * a.C + t0);
#pragma unroll
              for (int k4 = 0; k4 < P_HALF / 8; k4++)
                vrow[k4] = make_uint4(packed[4 * k4], packed[4 * k4 + 1], packed[4 * k4 + 2], packed[4 * k4 + 3]);
            }
          } else if constexpr (EPI == PEPI_SWIGLU) {
            // rows r < 64 hold the gate and rows r + 64 the up projection of feature r: both rows
            // land in the exchange buffer, then the thread of row r handles the first P_HALF/2
            // tokens of the warpgroup's slice and the thread of row r + 64 the rest
#pragma unroll
            for (int i = 0; i < P_HALF; i++) ys[r * P_YS_LD + i] = y[i];
            pf_sync_g(g);
            const int fr = r & 63, i0 = r < 64 ? 0 : P_HALF / 2;
            const int fcol = mt * 64 + fr;
#pragma unroll
            for (int k = 0; k < P_HALF / 2; k++) {
              const int i = i0 + k;
              const float gv = ys[fr * P_YS_LD + i], uv = ys[(fr + 64) * P_YS_LD + i];
              const float act = gv / (1.0f + expf(-gv)) * uv;
              const uint16_t hi = f2bf_bits(act);
              a.act_out[(size_t)(t0 + i) * a.ld_act + fcol] = hi;
              a.act_out[(size_t)(a.C + t0 + i) * a.ld_act + fcol] = f2bf_bits(act - bf2f(hi));
            }
          }
          pf_sync_g(g);  // ys / s_red reused by the next chunk
        }
       }
        if (tlast) tr[6] = globaltimer();
        tc_fence_before();
        pf_arrive(&acc_empty[buf]);
        if (nseg > 1 && et == 0) a.counters[u] = epoch + 1;  // read by the next launch only
      }
      f = fend;
    }
    tc_fence_before();
    pf_arrive(epi_done);
  }
  if (warp == 1) {
    // the epilogue warps' last TMEM reads are ordered before the dealloc by epi_done
    mbar_wait(epi_done, 0u, ST_EPI_WAIT, &g_status_prefill);
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// ------------------------------------------------- causal attention on tcgen05
// Within-prompt causal attention (kernels/prefill_full.py:64-70 with the mask of
// prefill_full.py:188 / cpu_layer_p :119): query t attends keys 0..t.
//
// One CTA = (32-query tile, kv head).  The 4 query heads of the kv head are packed into
// the MMA's M = 128 rows (row r = token qt*32 + r/4, head 4*kvh + r%4), so K and V are
// read once per group.  Per 128-key chunk:
//   S = Q K^T           tcgen05, M=128, N=128 keys, K=HD: Q enters as bf16 hi + lo rows
//                       (two MMAs into one TMEM accumulator: fp32-level q), K as bf16;
//   softmax             epilogue warps, thread r = row r: scale, causal mask, running max /
//                       sum (fp32), P = exp(S - m) written to shared memory as bf16 hi + lo
//                       in the 128-byte-swizzled K-major layout TMA would produce;
//   O_c = P V           tcgen05, M=128, N=HD, K=128 keys, B = V^T (written by the QKV
//                       epilogue into a scratch buffer so that it is K-major too);
//   o = o * corr + O_c  registers, fp32.
// Operands arrive by TMA: Q hi/lo boxes (64 d, 4 heads, 32 tokens), K boxes (64 d, 128
// keys) from the layer's cache, V^T boxes (64 keys, 128 d).  The output o / l goes out as
// the hi/lo bf16 operand of the O projection.
constexpr int kAQ = 32;               // query tokens per CTA (x 4 heads = 128 MMA rows)
constexpr int kAK = 128;              // keys per chunk
constexpr int kABox = 16384;          // one 128-row x 128-byte swizzled box
constexpr int kAttnG = 4;             // softmax / output warpgroups
constexpr int kAttnKpt = kAK / kAttnG;  // keys of a chunk, and output dims, per softmax thread
constexpr int kAttnT = 64 + 128 * kAttnG;  // TMA warp, MMA warp, the softmax warpgroups
// smem: Q, K, V^T, P boxes | barriers and TMEM slot (128 B) | row max / sum parts [2][kAttnG][128]
constexpr size_t kAttnTcSmem = 1024 + 12 * (size_t)kABox + 128 + 2 * kAttnG * 128 * 4;

__global__ void __launch_bounds__(kAttnT, 1) pf_attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                            const __grid_constant__ CUtensorMap tmK,
                                                            const __grid_constant__ CUtensorMap tmV, int C,
                                                            uint16_t* __restrict__ act_o, int ld_act) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = base;                  // [hi d0-63, hi d64-127, lo d0-63, lo d64-127]
  uint8_t* sK = sQ + 4 * kABox;        // [d0-63, d64-127]
  uint8_t* sV = sK + 2 * kABox;        // V^T: [keys 0-63, keys 64-127] of the chunk, rows = d
  uint8_t* sP = sV + 2 * kABox;        // [hi keys 0-63, hi keys 64-127, lo keys 0-63, lo keys 64-127]
  uint64_t* bar = (uint64_t*)(sP + 4 * kABox);
  uint64_t* q_full = bar + 0;
  uint64_t* k_full = bar + 1;          // the chunk's K boxes
  uint64_t* v_full = bar + 6;          // the chunk's V^T boxes
  uint64_t* s_full = bar + 2;
  uint64_t* p_full = bar + 3;
  uint64_t* o_full = bar + 4;
  uint64_t* epi_done = bar + 5;        // the softmax threads are past their last TMEM read
  uint32_t* tmem_slot = (uint32_t*)(bar + 8);
  float* red_m = (float*)(bar + 16);   // [kAttnG][128 rows] partial row max
  float* red_l = red_m + kAttnG * 128; // [kAttnG][128 rows] partial row sum

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, kvh = blockIdx.y;
  const int kend = qt * kAQ + kAQ;               // keys 0 .. kend-1 are needed
  const int nchunk = (kend + kAK - 1) / kAK;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(k_full, 1);
    mbar_init(v_full, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, 128 * kAttnG);
    mbar_init(o_full, 1);
    mbar_init(epi_done, 128 * kAttnG);
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);  // S: columns 0-127, O_c: 128-255
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 128;

  if (warp == 0) {
    if (lane == 0) {
      grid_dep_wait();  // q, K and V^T are written by the QKV GEMM
      mbar_arrive_expect_tx(q_full, 4 * kABox);
      for (int hl = 0; hl < 2; hl++)
        for (int bx = 0; bx < 2; bx++)
          tma_load_3d(sQ + (hl * 2 + bx) * kABox, &tmQ, q_full, bx * 64, kvh * 4, hl * C + qt * kAQ);
      // K of chunk c is loaded once S of chunk c-1 is done (during its softmax), V once P V of
      // chunk c-1 is done
      for (int c = 0; c < nchunk; c++) {
        if (c > 0 && !mbar_wait(s_full, (uint32_t)(c - 1) & 1u, ST_TMA_WAIT, &g_status_prefill)) break;
        mbar_arrive_expect_tx(k_full, 2 * kABox);
        for (int bx = 0; bx < 2; bx++) tma_load_3d(sK + bx * kABox, &tmK, k_full, bx * 64, c * kAK, kvh);
        if (c > 0 && !mbar_wait(o_full, (uint32_t)(c - 1) & 1u, ST_TMA_WAIT, &g_status_prefill)) break;
        mbar_arrive_expect_tx(v_full, 2 * kABox);
        for (int bx = 0; bx < 2; bx++) tma_load_3d(sV + bx * kABox, &tmV, v_full, c * kAK + bx * 64, 0, kvh);
      }
      grid_dep_launch();
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, 128);
      bool ok = mbar_wait(q_full, 0, ST_MMA_WAIT, &g_status_prefill);
      for (int c = 0; c < nchunk && ok; c++) {
        ok = mbar_wait(k_full, (uint32_t)c & 1u, ST_MMA_WAIT, &g_status_prefill);
        if (!ok) break;
        tc_fence_after();
        // S = (Qhi + Qlo) K^T over HD = 2 boxes x 4 K-steps
        for (int kk = 0; kk < 8; kk++) {
          const uint32_t off = (uint32_t)((kk >> 2) * kABox + (kk & 3) * 32);
          const uint64_t kd = sw128_kmajor_desc(smem_u32(sK) + off);
          umma_bf16(tS, sw128_kmajor_desc(smem_u32(sQ) + off), kd, idesc, kk != 0 ? 1u : 0u);
          umma_bf16(tS, sw128_kmajor_desc(smem_u32(sQ) + 2 * kABox + off), kd, idesc, 1u);
        }
        umma_commit(s_full);
        ok = mbar_wait(p_full, (uint32_t)c & 1u, ST_MMA_WAIT, &g_status_prefill) &&
             mbar_wait(v_full, (uint32_t)c & 1u, ST_MMA_WAIT, &g_status_prefill);
        if (!ok) break;
        tc_fence_after();
        // O_c = (Phi + Plo) V over the chunk's 128 keys = 2 boxes x 4 K-steps
        for (int kk = 0; kk < 8; kk++) {
          const uint32_t off = (uint32_t)((kk >> 2) * kABox + (kk & 3) * 32);
          const uint64_t vd = sw128_kmajor_desc(smem_u32(sV) + off);
          umma_bf16(tO, sw128_kmajor_desc(smem_u32(sP) + off), vd, idesc, kk != 0 ? 1u : 0u);
          umma_bf16(tO, sw128_kmajor_desc(smem_u32(sP) + 2 * kABox + off), vd, idesc, 1u);
        }
        umma_commit(o_full);
      }
      // TMEM is freed below only after every softmax thread has read its last accumulator
      mbar_wait(epi_done, 0u, ST_EPI_WAIT, &g_status_prefill);
      tc_fence_after();
    }
    __syncwarp();
    tmem_dealloc(tmem, 256);
  } else {
    // softmax / output warps: kAttnG warpgroups over the same 128 TMEM lanes.  Thread (h, r) owns
    // MMA row r = (token qt*32 + r/4, head 4*kvh + r%4) for keys kAttnKpt*h .. of every chunk and
    // the same output dims; the row's max and sum meet in shared memory.  More warpgroups shorten
    // the per-chunk softmax, which sits between the two MMAs of every chunk.
    const int h = (threadIdx.x - 64) >> 7;
    const int r = ((warp & 3) << 5) | lane;
    const int tok = qt * kAQ + (r >> 2);
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const float scale = 0.08838834764831845f;  // 1/sqrt(128)
    float o[kAttnKpt];
#pragma unroll
    for (int j = 0; j < kAttnKpt; j++) o[j] = 0.f;
    float m = -INFINITY, l = 0.f;
    uint8_t* prow = sP + (r >> 3) * 1024 + (r & 7) * 128;
    for (int c = 0; c < nchunk; c++) {
      if (!mbar_wait(s_full, (uint32_t)c & 1u, ST_EPI_WAIT, &g_status_prefill)) break;
      __syncwarp();
      tc_fence_after();
      float v[kAttnKpt];
      tmem_ld_32x32b_x32(tS + lane_base + h * kAttnKpt, v);
      float cm = -INFINITY;
#pragma unroll
      for (int j = 0; j < kAttnKpt; j++)
        if (c * kAK + h * kAttnKpt + j <= tok) cm = fmaxf(cm, v[j] * scale);
      red_m[h * 128 + r] = cm;
      asm volatile("bar.sync 1, %0;" ::"n"(128 * kAttnG) : "memory");
      float mx = red_m[r];
#pragma unroll
      for (int g2 = 1; g2 < kAttnG; g2++) mx = fmaxf(mx, red_m[g2 * 128 + r]);
      const float mnew = fmaxf(m, mx);
      const float corr = m == -INFINITY ? 0.f : expf(m - mnew);
      float lsum = 0.f;
#pragma unroll
      for (int g8 = 0; g8 < kAttnKpt / 8; g8++) {  // 8 keys = one 16-byte chunk of the swizzled row
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          float pp[2];
#pragma unroll
          for (int u = 0; u < 2; u++) {
            const int j = g8 * 8 + e + u;
            pp[u] = c * kAK + h * kAttnKpt + j <= tok ? expf(v[j] * scale - mnew) : 0.f;
            lsum += pp[u];
          }
          const uint16_t h0 = f2bf_bits(pp[0]), h1 = f2bf_bits(pp[1]);
          hw[e / 2] = (uint32_t)h0 | ((uint32_t)h1 << 16);
          lw[e / 2] = (uint32_t)f2bf_bits(pp[0] - bf2f(h0)) | ((uint32_t)f2bf_bits(pp[1] - bf2f(h1)) << 16);
        }
        const int key = h * kAttnKpt + g8 * 8;        // first key of these 8 within the chunk
        const int box = key >> 6;                      // 64 keys per 128-byte-wide box
        const int ch = ((key & 63) >> 3) ^ (r & 7);   // its swizzled 16-byte chunk in the row
        *reinterpret_cast<uint4*>(prow + box * kABox + (ch << 4)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(prow + (2 + box) * kABox + (ch << 4)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
      red_l[h * 128 + r] = lsum;
      fence_proxy_async_smem();  // P is read by the tensor cores
      tc_fence_before();
      pf_arrive(p_full);
      asm volatile("bar.sync 1, %0;" ::"n"(128 * kAttnG) : "memory");
      float ls = red_l[r];
#pragma unroll
      for (int g2 = 1; g2 < kAttnG; g2++) ls += red_l[g2 * 128 + r];
      l = l * corr + ls;
      m = mnew;
      if (!mbar_wait(o_full, (uint32_t)c & 1u, ST_EPI_WAIT, &g_status_prefill)) break;
      __syncwarp();
      tc_fence_after();
      float w[kAttnKpt];
      tmem_ld_32x32b_x32(tO + lane_base + h * kAttnKpt, w);
#pragma unroll
      for (int j = 0; j < kAttnKpt; j++) o[j] = fmaf(o[j], corr, w[j]);
    }
    tc_fence_before();
    pf_arrive(epi_done);
    const float inv_l = 1.0f / l;
    const int head = kvh * 4 + (r & 3);
    uint16_t* dh = act_o + (size_t)tok * ld_act + (size_t)head * 128 + h * kAttnKpt;
    uint16_t* dl = act_o + (size_t)(C + tok) * ld_act + (size_t)head * 128 + h * kAttnKpt;
#pragma unroll
    for (int d8 = 0; d8 < kAttnKpt / 8; d8++) {
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const float v0 = o[d8 * 8 + e] * inv_l, v1 = o[d8 * 8 + e + 1] * inv_l;
        const uint16_t h0 = f2bf_bits(v0), h1 = f2bf_bits(v1);
        hw[e / 2] = (uint32_t)h0 | ((uint32_t)h1 << 16);
        lw[e / 2] = (uint32_t)f2bf_bits(v0 - bf2f(h0)) | ((uint32_t)f2bf_bits(v1 - bf2f(h1)) << 16);
      }
      *reinterpret_cast<uint4*>(dh + d8 * 8) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(dl + d8 * 8) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
  }
}

// --------------------------------------------------------------- host side
static int pf_grid(long total) {
  const int g = num_sms();
  return total < g ? (int)total : g;
}

static int pf_maxseg(long units, long nkb, int grid) {
  const long total = units * nkb;
  int mx = 1;
  for (long u = 0; u < units; u++) {
    const int s = owner_of(u * nkb + nkb - 1, total, grid) - owner_of(u * nkb, total, grid) + 1;
    mx = s > mx ? s : mx;
  }
  return mx;
}

template <int EPI, int NT, int MT>
static int launch_pf(const void* W, int L, int layer, int N, int K, const void* act, int ld, PArgs a, cudaStream_t s) {
  RNGD_REQUIRE(K % PBK == 0 && N % (MT * PBM) == 0, "prefill GEMM: N=%d K=%d must be multiples of %d / 64", N, K,
               MT * PBM);
  RNGD_REQUIRE(a.C % NT == 0, "prefill GEMM: C=%d must be a multiple of %d", a.C, NT);
  CUtensorMap tw, tx;
  RNGD_TRY(get_weight_map_rows(W, L, N, K, MT * PBM, &tw));
  RNGD_TRY(get_operand_map(act, K, ld, 2 * a.C, NT, &tx));
  a.N = N;
  a.K = K;
  a.nkb = K / PBK;
  a.ntok = a.C / NT;
  const long units = (long)(N / (MT * PBM)) * a.ntok;
  a.total = (int)(units * a.nkb);
  const int grid = pf_grid(a.total);
  a.maxseg = pf_maxseg(units, a.nkb, grid);
  a.nunits = (int)units;
  a.layer = layer;
  if (RNGD_TRACE && a.trace == nullptr) a.trace = next_seq_trace();
  RNGD_REQUIRE(a.maxseg == 1 || (a.partial && a.counters), "prefill GEMM: split tiles need partial/counters");
  RNGD_REQUIRE(a.tag >= 1 && a.tag <= 15, "prefill GEMM: shape tag %d outside 1..15", a.tag);
  static std::atomic<unsigned long long> attr_set{0};
  RNGD_TRY(set_smem_limit_once((const void*)pfgemm_kernel<EPI, NT, MT>, (int)PCfg<NT, MT>::SMEM, &attr_set,
                               "cudaFuncSetAttribute(pfgemm)"));
  return launch_pdl(pfgemm_kernel<EPI, NT, MT>, dim3(grid), dim3(64 + P_EPI), PCfg<NT, MT>::SMEM, s, "pfgemm_kernel", tw,
                    tx, a);
}

// Two weight tiles per work unit halve the activation traffic per FLOP, but also halve
// the number of units; a GEMM with fewer units than SMs then splits every unit across
// several CTAs and its tail (partial sums, reduction) grows.  So: two tiles per unit when
// that still leaves at least one whole unit per SM.
static int pf_choose_mt(int N, int C) {
  const long pairs = (N / PBM) % 2 == 0 ? (long)(N / (2 * PBM)) * (C / 128) : 0;
  return pairs >= num_sms() ? 2 : 1;
}

template <int EPI>
static int launch_pf_any(const void* W, int L, int layer, int N, int K, const void* act, int ld, PArgs a,
                         cudaStream_t s) {
  // 128-token tiles (measured faster than 256-token tiles with fewer stages)
  if (pf_choose_mt(N, a.C) == 2) return launch_pf<EPI, 128, 2>(W, L, layer, N, K, act, ld, a, s);
  return launch_pf<EPI, 128, 1>(W, L, layer, N, K, act, ld, a, s);
}

// scratch of one GEMM shape
static void pf_shape_ws(int N, int K, int C, size_t* pf, size_t* ct) {
  const int NT = 128, MT = pf_choose_mt(N, C);  // as launch_pf_any chooses
  const long units = (long)(N / (MT * PBM)) * (C / NT), nkb = K / PBK;
  const int ms = pf_maxseg(units, nkb, pf_grid(units * nkb));
  *pf = ms > 1 ? (size_t)units * ms * MT * NT * PBM : 0;
  *ct = ms > 1 ? (size_t)units * (1 + ms) : 0;  // epochs, then flags
}

int launch_operand(const float* x, int ldx, int rows, int H, const float* w, void* act, int ld_act, float* ss,
                   unsigned long long* best, cudaStream_t s);
int launch_operand_ex(const float* x, int ldx, int rows, int H, const float* w, void* act, int ld_act, int lo_off,
                      float* ss, int ss_ld, unsigned long long* best, cudaStream_t s);
int launch_embed(const void* emb, const int32_t* toks, int H, int V, float* x, int B, cudaStream_t s);

}  // namespace rngd

using namespace rngd;

static int check_pio(const rngd_model_t* m, const rngd_prefill_io_t* io) {
  RNGD_REQUIRE(m && io, "prefill: null model or io");
  RNGD_REQUIRE(m->HD == 128 && m->NH == 4 * m->NKV, "prefill: kernels are built for HD=128, NH=4*NKV");
  RNGD_REQUIRE(m->H % 128 == 0 && (2 * m->M) % 128 == 0, "prefill: H and 2*M must be multiples of 128");
  RNGD_REQUIRE(io->C >= 128 && io->C % 128 == 0 && io->C <= 4096, "prefill: C=%d must be a multiple of 128", io->C);
  RNGD_REQUIRE(io->P >= 1 && io->P <= io->C && io->P <= io->S, "prefill: P=%d outside 1..min(C=%d, S=%d)", io->P,
               io->C, io->S);
  RNGD_REQUIRE(io->operand_lo == 0 || io->operand_lo == 1, "prefill: operand_lo=%d must be 0 or 1", io->operand_lo);
  RNGD_REQUIRE(io->kv && io->toks && io->x && io->q && io->act && io->act_o && io->act2 && io->ss && io->partial &&
                   io->counters,
               "prefill: null buffer");
  return RNGD_OK;
}

extern "C" int rngd_prefill_workspace(const rngd_model_t* m, int C, size_t* partial_floats, size_t* counters) {
  RNGD_REQUIRE(m && partial_floats && counters, "prefill_workspace: null argument");
  RNGD_REQUIRE(C >= 128 && C % 128 == 0, "prefill_workspace: C=%d must be a multiple of 128", C);
  const int QN = m->NH * m->HD, KN = m->NKV * m->HD;
  const int shapes[4][2] = {{QN + 2 * KN, m->H}, {m->H, QN}, {2 * m->M, m->H}, {m->H, m->M}};
  size_t pf = 0, ct = 0;
  for (auto& sh : shapes) {
    size_t p, c;
    pf_shape_ws(sh[0], sh[1], C, &p, &c);
    pf = pf > p ? pf : p;
    ct = ct > c ? ct : c;
  }
  *partial_floats = pf;
  *counters = ct;
  return RNGD_OK;
}

extern "C" int rngd_prefill_embed(const rngd_model_t* m, const rngd_prefill_io_t* io, rngd_stream_t stream) {
  RNGD_TRY(check_pio(m, io));
  cudaStream_t s = (cudaStream_t)stream;
  const int H = m->H, QN = m->NH * m->HD, ld = H > QN ? H : QN;
  RNGD_TRY(launch_embed(m->embed, io->toks, H, m->V, io->x, io->C, s));
  return launch_operand_ex(io->x, H, io->C, H, m->n1, io->act, ld, io->C, io->ss, io->C, nullptr, s);
}

// io->x already holds the residual stream (fp32 [C][H], written by the caller): layer0's first
// operand hi/lo(x * n1[layer0]) and the sums of squares (kernels/prefill_full.py:79-94:
// PrefillModel.forward receives x rather than token ids).
extern "C" int rngd_prefill_begin(const rngd_model_t* m, const rngd_prefill_io_t* io, int layer0,
                                  rngd_stream_t stream) {
  RNGD_TRY(check_pio(m, io));
  RNGD_REQUIRE(0 <= layer0 && layer0 < m->L, "prefill_begin: layer %d outside [0, %d)", layer0, m->L);
  const int H = m->H, QN = m->NH * m->HD, ld = H > QN ? H : QN;
  return launch_operand_ex(io->x, H, io->C, H, m->n1 + (size_t)layer0 * H, io->act, ld, io->C, io->ss, io->C,
                           nullptr, (cudaStream_t)stream);
}

// Causal attention of one layer on tcgen05 (pf_attn_tc_kernel): Q hi/lo from io->q, K from
// the layer's cache block, V^T from the act2 scratch, output into io->act_o.
static int launch_pf_attn(const rngd_model_t* m, const rngd_prefill_io_t* io, const uint16_t* kv, cudaStream_t s) {
  const int C = io->C, NKV = m->NKV, NH = m->NH;
  CUtensorMap tq, tk, tv;
  const uint64_t qd[3] = {128, (uint64_t)NH, (uint64_t)2 * C}, qs[2] = {256, (uint64_t)NH * 256};
  const uint32_t qb[3] = {64, 4, (uint32_t)kAQ};
  RNGD_TRY(get_map3_bf16(io->q, qd, qs, qb, &tq));
  // the cache block belongs to one request: encoded per call rather than cached
  const uint64_t kd[3] = {128, (uint64_t)io->S, (uint64_t)NKV}, ks[2] = {256, (uint64_t)io->S * 256};
  const uint32_t kb[3] = {64, (uint32_t)kAK, 1};
  RNGD_TRY(encode_tmap_bf16(&tk, kv, 3, kd, ks, kb));
  const uint64_t vd[3] = {(uint64_t)C, 128, (uint64_t)NKV}, vs[2] = {(uint64_t)C * 2, (uint64_t)C * 256};
  const uint32_t vb[3] = {64, 128, 1};
  RNGD_TRY(get_map3_bf16(io->act2, vd, vs, vb, &tv));
  static std::atomic<unsigned long long> attr_set{0};
  RNGD_TRY(set_smem_limit_once((const void*)pf_attn_tc_kernel, (int)kAttnTcSmem, &attr_set,
                               "cudaFuncSetAttribute(pf_attn_tc_kernel)"));
  return launch_pdl(pf_attn_tc_kernel, dim3(C / kAQ, NKV), dim3(kAttnT), kAttnTcSmem, s, "pf_attn_tc_kernel", tq, tk,
                    tv, C, (uint16_t*)io->act_o, NH * 128);
}

extern "C" int rngd_prefill_layers(const rngd_model_t* m, const rngd_prefill_io_t* io, int layer0, int layer1,
                                   rngd_stream_t stream) {
  RNGD_TRY(check_pio(m, io));
  RNGD_REQUIRE(0 <= layer0 && layer0 <= layer1 && layer1 <= m->L, "prefill: layers [%d, %d) outside [0, %d)",
               layer0, layer1, m->L);
  RNGD_REQUIRE(layer1 - layer0 <= io->kv_layers, "prefill: %d layers requested but the KV block holds %d",
               layer1 - layer0, io->kv_layers);
  cudaStream_t s = (cudaStream_t)stream;
  const int H = m->H, Mi = m->M, QN = m->NH * m->HD, KN = m->NKV * m->HD, NQKV = QN + 2 * KN;
  const int ld = H > QN ? H : QN;
  const size_t layer_elems = (size_t)2 * m->NKV * io->S * m->HD;
  for (int l = layer0; l < layer1; l++) {
    PArgs a = {};
    a.C = io->C;
    a.P = io->P;
    a.lo = io->operand_lo;
    a.partial = io->partial;
    a.counters = io->counters;
    a.ss_in = io->ss;
    a.ss_tiles = H / 128;
    a.eps = m->eps;
    a.inv_h = 1.0f / (float)H;
    a.inv = m->inv_freq; a.q = io->q; a.ldq = QN;
    a.kv = (uint16_t*)io->kv + (size_t)(l - layer0) * layer_elems;
    a.vt = (uint16_t*)io->act2;
    a.NH = m->NH; a.NKV = m->NKV; a.S = io->S;
    a.tag = 1;
    RNGD_TRY(launch_pf_any<PEPI_QKV>(m->wqkv, m->L, l, NQKV, H, io->act, ld, a, s));
    RNGD_TRY(launch_pf_attn(m, io, a.kv, s));
    a.x = io->x; a.ldx = H;
    a.w_next = m->n2 + (size_t)l * H; a.act_next = (uint16_t*)io->act; a.ld_next = ld; a.ss_out = io->ss;
    a.tag = 2;
    RNGD_TRY(launch_pf_any<PEPI_RESID>(m->wo, m->L, l, H, QN, io->act_o, QN, a, s));
    a.act_out = (uint16_t*)io->act2; a.ld_act = Mi;
    a.tag = 3;
    RNGD_TRY(launch_pf_any<PEPI_SWIGLU>(m->wgu, m->L, l, 2 * Mi, H, io->act, ld, a, s));
    a.w_next = l + 1 < m->L ? m->n1 + (size_t)(l + 1) * H : m->norm;
    a.tag = 4;
    RNGD_TRY(launch_pf_any<PEPI_RESID>(m->wd, m->L, l, H, Mi, io->act2, Mi, a, s));
  }
  return RNGD_OK;
}

extern "C" int rngd_tc_gemm_tokens_workspace(int N, int K, int C, size_t* partial_floats, size_t* counters) {
  RNGD_REQUIRE(partial_floats && counters, "tc_gemm_tokens_workspace: null argument");
  RNGD_REQUIRE(C >= 128 && C % 128 == 0, "tc_gemm_tokens_workspace: C=%d must be a multiple of 128", C);
  pf_shape_ws(N, K, C, partial_floats, counters);
  return RNGD_OK;
}

extern "C" int rngd_tc_gemm_tokens(const void* W, int N, int K, const float* X, int C, float* Y, void* act,
                                   float* partial, int32_t* counters, int prep, rngd_stream_t stream) {
  RNGD_REQUIRE(W && X && Y && act, "tc_gemm_tokens: null pointer");
  RNGD_REQUIRE(C >= 128 && C % 128 == 0, "tc_gemm_tokens: C=%d must be a multiple of 128", C);
  RNGD_REQUIRE(N % PBM == 0 && K % PBK == 0, "tc_gemm_tokens: need N %% 128 == 0 and K %% 64 == 0");
  cudaStream_t s = (cudaStream_t)stream;
  if (prep) RNGD_TRY(launch_operand_ex(X, K, C, K, nullptr, act, K, C, nullptr, 0, nullptr, s));
  PArgs a = {};
  a.C = C;
  a.P = C;
  a.partial = partial;
  a.counters = counters;
  a.x = Y;
  a.ldx = N;
  a.tag = 5;
  a.lo = 1;
  a.trace = RNGD_TRACE ? gemm_trace() : nullptr;
  return launch_pf_any<PEPI_RESID>(W, 1, 0, N, K, act, K, a, s);
}

int rngd::read_status_prefill(int* st, int reset) {
  RNGD_TRY(check_cuda(cudaMemcpyFromSymbol(st, g_status_prefill, sizeof(int)), "read prefill status"));
  if (reset) {
    const int zero = 0;
    RNGD_TRY(check_cuda(cudaMemcpyToSymbol(g_status_prefill, &zero, sizeof(int)), "reset prefill status"));
  }
  return RNGD_OK;
}
