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
// deterministic in-order reduction of tiles cut between CTAs.
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
constexpr int P_YS_LD = 33;

template <int NT>
struct PCfg {
  static constexpr int A_BYTES = PBM * PBK * 2;   // 16 KB weight tile
  static constexpr int B_BYTES = NT * PBK * 2;    // one token tile (hi or lo)
  static constexpr int STAGE = A_BYTES + 2 * B_BYTES;
  static constexpr int STAGES = NT == 256 ? 2 : 4;
  static constexpr int TMEM_COLS = 2 * NT;        // double-buffered accumulator
  static constexpr size_t BAR_BYTES = (2 * STAGES + 4) * 8;
  static constexpr size_t SMEM = 1024 + STAGES * STAGE + BAR_BYTES + 64 + NT * 4 + PBM * P_YS_LD * 4 + 4 * 32 * 4;
};

enum PEpi : int { PEPI_QKV = 0, PEPI_RESID = 1, PEPI_SWIGLU = 2 };

struct PArgs {
  int N, K, nkb, ntok, total, maxseg, layer;
  int C, P;
  float* partial;  // [units][maxseg][NT][128]
  int* counters;   // [units]
  const float* ss_in;  // [ss_tiles][C]
  int ss_tiles;
  float eps, inv_h;
  // QKV
  const float* inv;
  float* q;
  int ldq;
  uint16_t* kv;  // this layer's [2][NKV][S][HD]
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
};

__device__ __forceinline__ void pf_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
__device__ __forceinline__ void pf_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <int EPI, int NT>
__global__ void __launch_bounds__(192, 1) pfgemm_kernel(const __grid_constant__ CUtensorMap tmW,
                                                        const __grid_constant__ CUtensorMap tmX, PArgs a) {
  using Cfg = PCfg<NT>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(base + STAGES * Cfg::STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint32_t* tmem_slot = (uint32_t*)((uint8_t*)full + Cfg::BAR_BYTES);
  int* s_last = (int*)(tmem_slot + 1);
  float* s_scale = (float*)((uint8_t*)full + Cfg::BAR_BYTES + 64);   // [NT] RMS scale of the unit's tokens
  float* ys = s_scale + NT;                                          // [128][33]
  float* s_red = ys + PBM * P_YS_LD;                                  // [4][32]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  const long f0 = (long)cta * a.total / G, f1 = (long)(cta + 1) * a.total / G;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
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
        const int kb = (int)(f - u * a.nkb), mt = (int)(u / a.ntok);
        uint8_t* st = base + i * Cfg::STAGE;
        mbar_arrive_expect_tx(&full[i], Cfg::STAGE);
        tma_load_3d(st, &tmW, &full[i], kb * PBK, mt * PBM, a.layer);
      }
      grid_dep_wait();
      for (long i = 0; i < pre; i++) {
        const long f = f0 + i;
        const long u = f / a.nkb;
        const int kb = (int)(f - u * a.nkb), jt = (int)(u % a.ntok);
        uint8_t* st = base + i * Cfg::STAGE;
        tma_load_2d(st + Cfg::A_BYTES, &tmX, &full[i], kb * PBK, jt * NT);
        tma_load_2d(st + Cfg::A_BYTES + Cfg::B_BYTES, &tmX, &full[i], kb * PBK, a.C + jt * NT);
      }
      for (long i = pre; i < nk; i++) {
        const int s = (int)(i % STAGES);
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, ST_TMA_WAIT, &g_status_prefill)) break;
        const long f = f0 + i;
        const long u = f / a.nkb;
        const int kb = (int)(f - u * a.nkb), mt = (int)(u / a.ntok), jt = (int)(u % a.ntok);
        uint8_t* st = base + s * Cfg::STAGE;
        mbar_arrive_expect_tx(&full[s], Cfg::STAGE);
        tma_load_3d(st, &tmW, &full[s], kb * PBK, mt * PBM, a.layer);
        tma_load_2d(st + Cfg::A_BYTES, &tmX, &full[s], kb * PBK, jt * NT);
        tma_load_2d(st + Cfg::A_BYTES + Cfg::B_BYTES, &tmX, &full[s], kb * PBK, a.C + jt * NT);
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
        const uint32_t d = tmem + (uint32_t)(buf * NT);
        for (long g = f; g < fend && ok; g++, i++) {
          const int s = (int)(i % STAGES);
          const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
          ok = mbar_wait(&full[s], ph, ST_MMA_WAIT, &g_status_prefill);
          if (!ok) break;
          tc_fence_after();
          const uint32_t sa = smem_u32(base + s * Cfg::STAGE);
          const uint32_t sh = sa + Cfg::A_BYTES, sl = sh + Cfg::B_BYTES;
#pragma unroll
          for (int kk = 0; kk < PBK / 16; kk++) {
            const uint64_t ad = sw128_kmajor_desc(sa + kk * 32);
            umma_bf16(d, ad, sw128_kmajor_desc(sh + kk * 32), idesc, (g != f || kk != 0) ? 1u : 0u);
            umma_bf16(d, ad, sw128_kmajor_desc(sl + kk * 32), idesc, 1u);
          }
          umma_commit(&empty[s]);
        }
        umma_commit(&acc_full[buf]);
        f = fend;
      }
    }
    __syncwarp();
  } else {
    grid_dep_wait();
    const int r = ((warp & 3) << 5) | lane;
    const int et = threadIdx.x - 64;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    int seg = 0;
    for (long f = f0; f < f1; seg++) {
      const long u = f / a.nkb;
      const long ustart = u * a.nkb;
      const long fend = ustart + a.nkb < f1 ? ustart + a.nkb : f1;
      const int mt = (int)(u / a.ntok), jt = (int)(u % a.ntok);
      const int n = mt * PBM + r;
      const int buf = seg & 1;
      // RMS scales of this unit's NT tokens, read while the accumulator is still being built:
      // token jt*NT + i's sum over the ss tiles in tile order, loads batched 16 at a time
      if (EPI != PEPI_RESID && a.ss_in != nullptr) {
        for (int i = et; i < NT; i += 128) {
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
        pf_sync();
      }
      mbar_wait(&acc_full[buf], (uint32_t)(seg >> 1) & 1u, ST_EPI_WAIT, &g_status_prefill);
      __syncwarp();
      tc_fence_after();
      const int first = owner_of(ustart, a.total, G), last = owner_of(ustart + a.nkb - 1, a.total, G);
      const int nseg = last - first + 1;
      const uint32_t tbase = tmem + lane_base + (uint32_t)(buf * NT);
      bool run = true;
      if (nseg > 1) {
        const int slot = cta - first;
        float* pdst = a.partial + ((size_t)u * a.maxseg + slot) * NT * PBM;
        for (int cc = 0; cc < NT / 32; cc++) {
          float v[32];
          tmem_ld_32x32b_x32(tbase + cc * 32, v);
#pragma unroll
          for (int i = 0; i < 32; i++) __stcg(pdst + (size_t)(cc * 32 + i) * PBM + r, v[i]);
        }
        tc_fence_before();
        pf_arrive(&acc_empty[buf]);
        __threadfence();
        pf_sync();
        if (et == 0) *s_last = (atomicAdd(&a.counters[u], 1) == nseg - 1);
        pf_sync();
        run = *s_last != 0;
        if (run) __threadfence();
      }
      if (run) {
        for (int cc = 0; cc < NT / 32; cc++) {
          float y[32];
          if (nseg > 1) {
#pragma unroll
            for (int i = 0; i < 32; i++) y[i] = 0.f;
            for (int sl = 0; sl < nseg; sl++) {
              const float* src = a.partial + ((size_t)u * a.maxseg + sl) * NT * PBM + (size_t)(cc * 32) * PBM + r;
#pragma unroll
              for (int i = 0; i < 32; i++) y[i] += __ldcg(src + (size_t)i * PBM);
            }
          } else {
            tmem_ld_32x32b_x32(tbase + cc * 32, y);
          }
          const int t0 = jt * NT + cc * 32;  // first token of the chunk
          if (EPI != PEPI_RESID && a.ss_in != nullptr) {
#pragma unroll
            for (int i = 0; i < 32; i++) y[i] *= s_scale[cc * 32 + i];
          }
          if constexpr (EPI == PEPI_RESID) {
            float xo[32];  // all 32 residual loads in flight before the first store
#pragma unroll
            for (int i = 0; i < 32; i++) xo[i] = a.x[(size_t)(t0 + i) * a.ldx + n];
#pragma unroll
            for (int i = 0; i < 32; i++) {
              const float xn = xo[i] + y[i];
              a.x[(size_t)(t0 + i) * a.ldx + n] = xn;
              y[i] = xn;
            }
            if (a.act_next != nullptr) {
              const float w = a.w_next[n];
#pragma unroll
              for (int i = 0; i < 32; i++) {
                const float h = y[i] * w;
                const uint16_t hi = f2bf_bits(h);
                a.act_next[(size_t)(t0 + i) * a.ld_next + n] = hi;
                a.act_next[(size_t)(a.C + t0 + i) * a.ld_next + n] = f2bf_bits(h - bf2f(hi));
              }
#pragma unroll
              for (int i = 0; i < 32; i++) {
                const float sq = warp_sum(y[i] * y[i]);
                if (lane == 0) s_red[(warp & 3) * 32 + i] = sq;
              }
              pf_sync();
              if (et < 32)
                a.ss_out[(size_t)mt * a.C + t0 + et] =
                    (s_red[et] + s_red[32 + et]) + (s_red[64 + et] + s_red[96 + et]);
            }
          } else if constexpr (EPI == PEPI_QKV) {
#pragma unroll
            for (int i = 0; i < 32; i++) ys[r * P_YS_LD + i] = y[i];
            pf_sync();
            const int head = mt;
            const int idx = r & 63;
            const bool lo_half = r < 64;
            const int partner = r ^ 64;
            if (head < a.NH + a.NKV) {
              const float invf = a.inv[idx];
#pragma unroll 8
              for (int i = 0; i < 32; i++) {
                const int t = t0 + i;
                float sn, cs;
                sincosf((float)t * invf, &sn, &cs);
                const float other = ys[partner * P_YS_LD + i];
                const float o = lo_half ? y[i] * cs - other * sn : y[i] * cs + other * sn;
                if (head < a.NH) {
                  a.q[(size_t)t * a.ldq + n] = o;
                } else if (t < a.P) {
                  a.kv[(((size_t)(head - a.NH)) * a.S + t) * 128 + r] = f2bf_bits(o);
                }
              }
            } else {
              const int vh = head - a.NH - a.NKV;
#pragma unroll 8
              for (int i = 0; i < 32; i++) {
                const int t = t0 + i;
                if (t < a.P) a.kv[(((size_t)(a.NKV + vh)) * a.S + t) * 128 + r] = f2bf_bits(y[i]);
              }
            }
          } else if constexpr (EPI == PEPI_SWIGLU) {
#pragma unroll
            for (int i = 0; i < 32; i++) ys[r * P_YS_LD + i] = y[i];
            pf_sync();
            if (r < 64) {
              const int fcol = mt * 64 + r;
#pragma unroll 8
              for (int i = 0; i < 32; i++) {
                const float g = y[i], uu = ys[(r + 64) * P_YS_LD + i];
                const float act = g / (1.0f + expf(-g)) * uu;
                const uint16_t hi = f2bf_bits(act);
                a.act_out[(size_t)(t0 + i) * a.ld_act + fcol] = hi;
                a.act_out[(size_t)(a.C + t0 + i) * a.ld_act + fcol] = f2bf_bits(act - bf2f(hi));
              }
            }
          }
          pf_sync();  // ys / s_scale / s_red reused by the next chunk
        }
        if (nseg > 1) {
          if (et == 0) a.counters[u] = 0;
        } else {
          tc_fence_before();
          pf_arrive(&acc_empty[buf]);
        }
      }
      f = fend;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, Cfg::TMEM_COLS);
}

// ------------------------------------------------------- causal attention
// Within-prompt causal attention (kernels/prefill_full.py:64-70 with the mask of
// prefill_full.py:188 / cpu_layer_p :119): query t attends keys 0..t.  One CTA =
// (32-query tile, query head); 4 threads per query row, 32 dims each.  Keys and
// values are read from the bf16 cache this layer just emitted (the values decode
// will see), staged 32 keys at a time into padded shared memory with cp.async.
// fp32 online softmax; the result goes out as the hi/lo operand of the O GEMM.
constexpr int kPQT = 32, kPKC = 32, kPRow = 272;

__device__ __forceinline__ void pf_cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}

__global__ void __launch_bounds__(128) pf_attn_kernel(const float* __restrict__ q, int ldq,
                                                      const uint16_t* __restrict__ kv, int NH, int NKV, int S,
                                                      int C, uint16_t* __restrict__ act_o, int ld_act) {
  __shared__ __align__(16) uint8_t sK[kPKC * kPRow];
  __shared__ __align__(16) uint8_t sV[kPKC * kPRow];
  grid_dep_wait();
  grid_dep_launch();
  const int qt = blockIdx.x, h = blockIdx.y, t = threadIdx.x;
  const int row = t >> 2, part = t & 3;  // query row within the tile, 32-dim slice
  const int tq = qt * kPQT + row;        // query token
  const int kvh = h / (NH / NKV);
  const uint8_t* kg = (const uint8_t*)(kv + ((size_t)kvh * S) * 128);
  const uint8_t* vg = (const uint8_t*)(kv + ((size_t)(NKV + kvh) * S) * 128);
  const float scale = 0.08838834764831845f;  // 1/sqrt(128)
  float qv[32], o[32];
  const float* qp = q + (size_t)tq * ldq + (size_t)h * 128 + part * 32;
#pragma unroll
  for (int d = 0; d < 32; d++) {
    qv[d] = qp[d];
    o[d] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const int kend = qt * kPQT + kPQT;  // keys needed by the tile: 0 .. kend-1
  for (int k0 = 0; k0 < kend; k0 += kPKC) {
    __syncthreads();  // the previous chunk is consumed
    for (int i = t; i < kPKC * 16; i += 128) {
      const int j = i >> 4, c16 = (i & 15) * 16;
      pf_cp_async16(sK + j * kPRow + c16, kg + (size_t)(k0 + j) * 256 + c16);
      pf_cp_async16(sV + j * kPRow + c16, vg + (size_t)(k0 + j) * 256 + c16);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    float sc[kPKC];
    float cmax = -INFINITY;
#pragma unroll 4
    for (int j = 0; j < kPKC; j++) {
      const uint8_t* kr = sK + j * kPRow + part * 64;
      float acc = 0.f;
#pragma unroll
      for (int v4 = 0; v4 < 4; v4++) {
        float kf[8];
        unpack8(*reinterpret_cast<const uint4*>(kr + v4 * 16), kf);
#pragma unroll
        for (int e = 0; e < 8; e++) acc = fmaf(qv[v4 * 8 + e], kf[e], acc);
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      const float s = (k0 + j <= tq) ? acc * scale : -INFINITY;
      sc[j] = s;
      cmax = fmaxf(cmax, s);
    }
    const float mnew = fmaxf(m, cmax);
    if (mnew != -INFINITY) {
      const float corr = expf(m - mnew);
      l *= corr;
#pragma unroll
      for (int d = 0; d < 32; d++) o[d] *= corr;
      m = mnew;
#pragma unroll 4
      for (int j = 0; j < kPKC; j++) {
        if (sc[j] == -INFINITY) continue;
        const float p = expf(sc[j] - m);
        l += p;
        const uint8_t* vr = sV + j * kPRow + part * 64;
#pragma unroll
        for (int v4 = 0; v4 < 4; v4++) {
          float vf[8];
          unpack8(*reinterpret_cast<const uint4*>(vr + v4 * 16), vf);
#pragma unroll
          for (int e = 0; e < 8; e++) o[v4 * 8 + e] = fmaf(p, vf[e], o[v4 * 8 + e]);
        }
      }
    }
  }
  const float inv_l = 1.0f / l;
  uint16_t* dh = act_o + (size_t)tq * ld_act + (size_t)h * 128 + part * 32;
  uint16_t* dl = act_o + (size_t)(C + tq) * ld_act + (size_t)h * 128 + part * 32;
#pragma unroll
  for (int d = 0; d < 32; d++) {
    const float v = o[d] * inv_l;
    const uint16_t hi = f2bf_bits(v);
    dh[d] = hi;
    dl[d] = f2bf_bits(v - bf2f(hi));
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

template <int EPI, int NT>
static int launch_pf(const void* W, int L, int layer, int N, int K, const void* act, int ld, PArgs a, cudaStream_t s) {
  RNGD_REQUIRE(K % PBK == 0 && N % PBM == 0, "prefill GEMM: N=%d K=%d must be multiples of 128 / 64", N, K);
  RNGD_REQUIRE(a.C % NT == 0, "prefill GEMM: C=%d must be a multiple of %d", a.C, NT);
  CUtensorMap tw, tx;
  RNGD_TRY(get_weight_map(W, L, N, K, &tw));
  RNGD_TRY(get_operand_map(act, K, ld, 2 * a.C, NT, &tx));
  a.N = N;
  a.K = K;
  a.nkb = K / PBK;
  a.ntok = a.C / NT;
  const long units = (long)(N / PBM) * a.ntok;
  a.total = (int)(units * a.nkb);
  const int grid = pf_grid(a.total);
  a.maxseg = pf_maxseg(units, a.nkb, grid);
  a.layer = layer;
  RNGD_REQUIRE(a.maxseg == 1 || (a.partial && a.counters), "prefill GEMM: split tiles need partial/counters");
  static std::atomic<unsigned long long> attr_set{0};
  RNGD_TRY(set_smem_limit_once((const void*)pfgemm_kernel<EPI, NT>, (int)PCfg<NT>::SMEM, &attr_set,
                               "cudaFuncSetAttribute(pfgemm)"));
  return launch_pdl(pfgemm_kernel<EPI, NT>, dim3(grid), dim3(192), PCfg<NT>::SMEM, s, "pfgemm_kernel", tw, tx, a);
}

template <int EPI>
static int launch_pf_any(const void* W, int L, int layer, int N, int K, const void* act, int ld, PArgs a,
                         cudaStream_t s) {
  // 128-token tiles: a 48 KB stage (weights + hi + lo) leaves room for 4 stages in flight,
  // which measured faster than 256-token tiles with 2 stages at every bucket width
  return launch_pf<EPI, 128>(W, L, layer, N, K, act, ld, a, s);
}

// scratch of one GEMM shape
static void pf_shape_ws(int N, int K, int C, size_t* pf, size_t* ct) {
  const int NT = 128;
  const long units = (long)(N / PBM) * (C / NT), nkb = K / PBK;
  const int ms = pf_maxseg(units, nkb, pf_grid(units * nkb));
  *pf = ms > 1 ? (size_t)units * ms * NT * PBM : 0;
  *ct = ms > 1 ? (size_t)units : 0;
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
    a.partial = io->partial;
    a.counters = io->counters;
    a.ss_in = io->ss;
    a.ss_tiles = H / 128;
    a.eps = m->eps;
    a.inv_h = 1.0f / (float)H;
    a.inv = m->inv_freq; a.q = io->q; a.ldq = QN;
    a.kv = (uint16_t*)io->kv + (size_t)(l - layer0) * layer_elems;
    a.NH = m->NH; a.NKV = m->NKV; a.S = io->S;
    RNGD_TRY(launch_pf_any<PEPI_QKV>(m->wqkv, m->L, l, NQKV, H, io->act, ld, a, s));
    RNGD_TRY(launch_pdl(pf_attn_kernel, dim3(io->C / kPQT, m->NH), dim3(128), 0, s, "pf_attn_kernel",
                        (const float*)io->q, QN, (const uint16_t*)a.kv, m->NH, m->NKV, io->S, io->C,
                        (uint16_t*)io->act_o, QN));
    a.x = io->x; a.ldx = H;
    a.w_next = m->n2 + (size_t)l * H; a.act_next = (uint16_t*)io->act; a.ld_next = ld; a.ss_out = io->ss;
    RNGD_TRY(launch_pf_any<PEPI_RESID>(m->wo, m->L, l, H, QN, io->act_o, QN, a, s));
    a.act_out = (uint16_t*)io->act2; a.ld_act = Mi;
    RNGD_TRY(launch_pf_any<PEPI_SWIGLU>(m->wgu, m->L, l, 2 * Mi, H, io->act, ld, a, s));
    a.w_next = l + 1 < m->L ? m->n1 + (size_t)(l + 1) * H : m->norm;
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
