// Batched decode step for B <= 16 streams at independent positions.
//
// Replaces the reference's compiled decode graph (DecodeLayer.forward,
// src/rngd_pd/kernels/decode_batch.py:73-91) and its lm_head + host argmax
// (src/rngd_pd/engines/decode_batch.py:103-171).  The residual stream and all
// accumulations stay fp32; only weights and the KV cache are bf16 (the cache
// is written rounded to nearest even, exactly as the test oracle models it).
//
// Per layer:  rmsnorm -> QKV GEMV -> RoPE + KV append -> split-S attention
//             -> O GEMV (+= residual) -> rmsnorm -> gate/up GEMV -> SwiGLU
//             -> down GEMV (+= residual)
// HBM-bound: the GEMVs stream 436 MB of weights per layer; activations are a
// few hundred KB and stay in L1/L2.
#include <mutex>

#include "tc.cuh"

namespace rngd {

// ------------------------------------------------------------------ GEMV
// One warp owns R consecutive rows; each lane streams 16-byte vectors of every
// row at k = lane*8 + 256*i and keeps R*BT fp32 partial sums, reduced across
// the warp at the end.  Activation rows are read through L1 (shared by the
// CTA's 8 warps); weights bypass L1 (read once).
template <int BT, int R>
__global__ void __launch_bounds__(256) gemv_kernel(const uint16_t* __restrict__ W, int N, int K,
                                                   const float* __restrict__ X, int ldx, int B,
                                                   float* __restrict__ Y, int ldy, int accumulate) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows_per_cta = 8 * R;
  for (int n0 = blockIdx.x * rows_per_cta + warp * R; n0 < N; n0 += gridDim.x * rows_per_cta) {
    float acc[R][BT];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int b = 0; b < BT; b++) acc[r][b] = 0.f;
#pragma unroll 2
    for (int k = lane * 8; k < K; k += 256) {
      float w[R][8];
#pragma unroll
      for (int r = 0; r < R; r++) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (n0 + r < N) v = ldg_nc_v4(W + (size_t)(n0 + r) * K + k);
        unpack8(v, w[r]);
      }
#pragma unroll
      for (int b = 0; b < BT; b++) {
        if (b >= B) break;  // rows past B are neither read nor written
        const float4 x0 = __ldg(reinterpret_cast<const float4*>(X + (size_t)b * ldx + k));
        const float4 x1 = __ldg(reinterpret_cast<const float4*>(X + (size_t)b * ldx + k + 4));
#pragma unroll
        for (int r = 0; r < R; r++) {
          float a = acc[r][b];
          a = fmaf(w[r][0], x0.x, a); a = fmaf(w[r][1], x0.y, a);
          a = fmaf(w[r][2], x0.z, a); a = fmaf(w[r][3], x0.w, a);
          a = fmaf(w[r][4], x1.x, a); a = fmaf(w[r][5], x1.y, a);
          a = fmaf(w[r][6], x1.z, a); a = fmaf(w[r][7], x1.w, a);
          acc[r][b] = a;
        }
      }
    }
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int b = 0; b < BT; b++) {
        float v = warp_sum(acc[r][b]);
        // spread the stores over the lanes of the warp
        if (lane == ((r * BT + b) & 31) && n0 + r < N && b < B) {
          float* y = Y + (size_t)b * ldy + n0 + r;
          *y = accumulate ? *y + v : v;
        }
      }
  }
}

template <int BT>
static int launch_gemv_bt(const uint16_t* W, int N, int K, const float* X, int ldx, int B, float* Y,
                          int ldy, int accumulate, cudaStream_t s) {
  constexpr int R = BT >= 8 ? 2 : 4;
  int rows = 8 * R;
  int blocks = (N + rows - 1) / rows;
  gemv_kernel<BT, R><<<blocks, 256, 0, s>>>(W, N, K, X, ldx, B, Y, ldy, accumulate);
  return check_launch("gemv_kernel");
}

int launch_gemv(const void* W, int N, int K, const float* X, int ldx, int B, float* Y, int ldy,
                int accumulate, cudaStream_t s) {
  RNGD_REQUIRE(W && X && Y, "gemv: null pointer");
  RNGD_REQUIRE(N > 0 && K > 0 && K % 8 == 0, "gemv: need N > 0 and K %% 8 == 0 (N=%d K=%d)", N, K);
  RNGD_REQUIRE(B >= 1 && B <= 16, "gemv: batch %d outside 1..16", B);
  RNGD_REQUIRE(ldx % 4 == 0 && ldx >= K, "gemv: ldx %d must be >= K and a multiple of 4", ldx);
  const uint16_t* w = (const uint16_t*)W;
  if (B <= 1) return launch_gemv_bt<1>(w, N, K, X, ldx, B, Y, ldy, accumulate, s);
  if (B <= 2) return launch_gemv_bt<2>(w, N, K, X, ldx, B, Y, ldy, accumulate, s);
  if (B <= 4) return launch_gemv_bt<4>(w, N, K, X, ldx, B, Y, ldy, accumulate, s);
  if (B <= 8) return launch_gemv_bt<8>(w, N, K, X, ldx, B, Y, ldy, accumulate, s);
  return launch_gemv_bt<16>(w, N, K, X, ldx, B, Y, ldy, accumulate, s);
}

// -------------------------------------------------------------- rmsnorm
// out = x * (1 / sqrt(mean(x^2) + eps)) * w   (kernels/decode_batch.py:130)
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* __restrict__ x, int H,
                                                      const float* __restrict__ w, float eps,
                                                      float* __restrict__ out) {
  __shared__ float red[8];
  const float* xr = x + (size_t)blockIdx.x * H;
  float s = 0.f;
  for (int k = threadIdx.x; k < H; k += 256) s = fmaf(xr[k], xr[k], s);
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < 8 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = 1.0f / sqrtf(t / (float)H + eps);
  }
  __syncthreads();
  const float inv = red[0];
  float* o = out + (size_t)blockIdx.x * H;
  for (int k = threadIdx.x; k < H; k += 256) o[k] = xr[k] * inv * w[k];
}

int launch_rmsnorm(const float* x, int R, int H, const float* w, float eps, float* out, cudaStream_t s) {
  RNGD_REQUIRE(x && w && out && R > 0 && H > 0, "rmsnorm: bad arguments");
  rmsnorm_kernel<<<R, 256, 0, s>>>(x, H, w, eps, out);
  return check_launch("rmsnorm_kernel");
}

// ------------------------------------------------------ RoPE + KV append
// HF rotate-half on q and k at pos[b] (kernels/decode_batch.py:133-142), angles
// fp32 = float(pos) * inv_freq (engines/decode_batch.py:248-253); k and v are
// rounded to bf16 and written into lane b at pos[b] (the one-hot injection of
// kernels/decode_batch.py:81-82, as a store).
// grid (B, NH + 2*NKV), block HD/2.
__global__ void rope_kv_kernel(const float* __restrict__ qkv, int ldqkv, const int32_t* __restrict__ pos,
                               const float* __restrict__ inv, float* __restrict__ q, int ldq,
                               uint16_t* __restrict__ kc, uint16_t* __restrict__ vc, int NH, int NKV,
                               int HD, int S) {
  const int b = blockIdx.x, hd = blockIdx.y, i = threadIdx.x, half = HD >> 1;
  const int p = pos[b];
  if (p < 0 || p >= S) return;  // the host validates positions; never write outside the lane
  const float* src = qkv + (size_t)b * ldqkv + (size_t)hd * HD;
  const float a = src[i], c = src[i + half];
  if (hd < NH + NKV) {
    const float ang = (float)p * inv[i];
    float sn, cs;
    sincosf(ang, &sn, &cs);
    const float r0 = a * cs - c * sn, r1 = c * cs + a * sn;
    if (hd < NH) {
      float* dq = q + (size_t)b * ldq + (size_t)hd * HD;
      dq[i] = r0;
      dq[i + half] = r1;
    } else {
      uint16_t* dk = kc + (((size_t)b * NKV + (hd - NH)) * S + p) * HD;
      dk[i] = f2bf_bits(r0);
      dk[i + half] = f2bf_bits(r1);
    }
  } else {
    uint16_t* dv = vc + (((size_t)b * NKV + (hd - NH - NKV)) * S + p) * HD;
    dv[i] = f2bf_bits(a);
    dv[i + half] = f2bf_bits(c);
  }
}

// ------------------------------------------------------------ attention
// Split-S flash decoding with a fixed 128-position chunk (independent of B and
// of the other lanes, so a stream's result does not depend on who it is
// batched with).  One CTA = (chunk, kv head, stream) and the G=4 query heads
// that share the kv head.  Positions > pos[b] are skipped; the reference masks
// them with -1e4 (kernels/decode_batch.py:153), which gives them probability
// exactly 0 in fp32 as well.
constexpr int kChunk = 128;
constexpr int kG = 4;
constexpr int kHD = 128;

constexpr int kRowBytes = 272;  // smem pitch of a staged K/V row: 256 B + 16 B pad (bank-conflict free)
constexpr int kPhlLd = kRowBytes / 2;  // bf16 pitch of the P operand rows (same bank spread as K/V)
// smem: K rows | V rows | P operand [8][kPhlLd] bf16 | per-warp max and sum [2][kG][8]
constexpr size_t kAttnSmem = 2 * kChunk * kRowBytes + 8 * kRowBytes + 2 * kG * 8 * 4 + 128;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}

// Warp-level bf16 tensor-core pieces (16x8x16 tiles, fp32 accumulation) for the small
// decode-attention contractions: 4 query heads x {hi, lo} bf16 halves make the 8 columns.
__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void ldsm_x4_t(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// hi or lo bf16 half (part 0 / 1) of two fp32 values, packed low index first
__device__ __forceinline__ uint32_t pack_hilo(float x0, float x1, int part) {
  const uint16_t h0 = f2bf_bits(x0), h1 = f2bf_bits(x1);
  if (part == 0) return (uint32_t)h0 | ((uint32_t)h1 << 16);
  return (uint32_t)f2bf_bits(x0 - bf2f(h0)) | ((uint32_t)f2bf_bits(x1 - bf2f(h1)) << 16);
}

__device__ int g_status_attn = 0;  // this file's bounded-wait status word

// One 64-bit {value, flag} word of a fused-attention chunk record; single-copy atomic, so a
// reader that sees the flag sees the value stored with it.
__device__ __forceinline__ void st_rec(unsigned long long* p, float v, uint32_t flag) {
  const unsigned long long w = ((unsigned long long)flag << 32) | __float_as_uint(v);
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_rec(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

constexpr int kRecChunks = 3;  // chunk records the fused combine reads per poll round

constexpr int kAttnThreads = 256;  // two halves of 128 threads, one per pair of query heads

// One CTA = (128-position chunk, kv head, stream) and the G=4 query heads of the kv head;
// thread t works on query heads 2*(t/128), 2*(t/128)+1 at position / dimension t % 128.
// The chunk's K rows, then its V rows, are staged into shared memory with cp.async (all loads
// in flight at once); the scores (one position per thread) and softmax statistics run as soon
// as K has landed, P.V once V has.  Every per-head sum runs in the same order whatever the
// thread split, so both forms below give the same bits.
//
// FUSED = false writes a partial record (o[HD], m, l per head) for attn_combine_kernel.
// FUSED = true (the decode step, launched right after the QKV GEMM that appends K/V at
// pos[b]):
//  * rows before pos[b] were written by earlier steps and every kernel before the QKV GEMM
//    has completed once this grid is running (the GEMM signals its dependants only after its
//    own dependency wait), so they are staged BEFORE the wait, overlapping the GEMM's tail;
//    the row at pos[b] and q are read after it;
//  * the combine runs in the same grid: chunks 1.. store their records as {value, flag} words,
//    flag = epoch of (stream, kv head) + 1; chunk 0 (the lowest CTA index of the group, so it
//    only ever waits on CTAs dispatched after it) polls them with a bounded wait, combines
//    every chunk in chunk order exactly as attn_combine_kernel does, writes the hi/lo operand
//    of the O projection and advances the epoch, so records of earlier launches (older
//    epochs) never read as ready and nothing needs clearing.
template <bool FUSED>
__device__ __forceinline__ void attn_chunk(const float* __restrict__ q, int ldq, const uint16_t* __restrict__ kc,
                                           const uint16_t* __restrict__ vc, const int32_t* __restrict__ pos,
                                           const int32_t* __restrict__ lanes, int NH, int NKV, int S,
                                           float* __restrict__ part,
                                           unsigned long long* __restrict__ recw, int* __restrict__ epochs,
                                           uint16_t* __restrict__ act, int ld_act) {
  extern __shared__ __align__(16) uint8_t attn_smem[];
  uint8_t* sK = attn_smem;
  uint8_t* sV = sK + kChunk * kRowBytes;
  uint16_t* phl = (uint16_t*)(sV + kChunk * kRowBytes);  // [8][kPhlLd]: p hi (heads 0-3), p lo (0-3)
  float* red_max = (float*)(phl + 8 * kPhlLd);           // [kG][8 warps]
  float* red_sum = red_max + kG * 8;                     // [kG][8 warps]
  float* ored = (float*)sK;                              // [kG][kHD], reuses the K rows after the scores

  const int c = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z, t = threadIdx.x;
  const int hp = t >> 7, tt = t & 127;             // head pair, position / dimension
  const int lane = t & 31;
  const int nchunk = gridDim.x;
  const int PS = kHD + 2;  // partial record: o[HD], m, l
  const int s0 = c * kChunk;
  const int lane_b = lanes != nullptr ? lanes[b] : b;  // the cache lane this stream reads
  const size_t head_base = ((size_t)lane_b * NKV + kvh) * (size_t)S * kHD;
  const uint8_t* kg = (const uint8_t*)(kc + head_base + (size_t)s0 * kHD);
  const uint8_t* vg = (const uint8_t*)(vc + head_base + (size_t)s0 * kHD);
  int P, n, old = 0;  // positions < P are attended; rows [0, old) of the chunk staged early
  if constexpr (FUSED) {
    const int pb = pos[b];
    P = min(pb + 1, S);
    n = min(kChunk, P - s0);
    if (n <= 0) return;  // no positions in this chunk: chunk 0 reads only chunks that hold some
    // rows this step may write: from pos[b] on; with a lane map, from the smallest position of
    // any stream (streams sharing a lane append to it in this same step)
    int fresh = pb;
    if (lanes != nullptr)
      for (int bb = 0; bb < (int)gridDim.z; bb++) fresh = min(fresh, pos[bb]);
    old = max(0, min(n, fresh - s0));
    for (int i = t; i < old * 16; i += kAttnThreads) {
      const int j = i >> 4, c16 = (i & 15) * 16;
      cp_async16(sK + j * kRowBytes + c16, kg + (size_t)j * 256 + c16);
      cp_async16(sV + j * kRowBytes + c16, vg + (size_t)j * 256 + c16);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  grid_dep_wait();
  // the next kernel (a weight-streaming GEMM) may start its prologue: at once here, after this
  // CTA's K/V rows have landed in the fused form, so its weight prefetch does not compete with them
  if constexpr (!FUSED) grid_dep_launch();
  float* rec0 = nullptr;
  int epoch = 0;
  if constexpr (FUSED) {
    epoch = __ldcg(epochs + (size_t)b * NKV + kvh);
  } else {
    P = min(pos[b] + 1, S);
    n = min(kChunk, P - s0);
    rec0 = part + (((size_t)b * NH + kvh * kG) * nchunk + c) * PS;
    if (n <= 0) {
      if (t < kG) {
        float* rec = rec0 + (size_t)t * nchunk * PS;
        rec[kHD] = -INFINITY;
        rec[kHD + 1] = 0.f;
      }
      return;
    }
  }
  for (int i = old * 16 + t; i < n * 16; i += kAttnThreads) {
    const int j = i >> 4, c16 = (i & 15) * 16;
    cp_async16(sK + j * kRowBytes + c16, kg + (size_t)j * 256 + c16);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int i = old * 16 + t; i < n * 16; i += kAttnThreads) {
    const int j = i >> 4, c16 = (i & 15) * 16;
    cp_async16(sV + j * kRowBytes + c16, vg + (size_t)j * 256 + c16);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  const float scale = 0.08838834764831845f;  // 1/sqrt(128) in fp32
  const int warp = t >> 5, gid = lane >> 2, tig = lane & 3;
  const int nt = (n + 15) >> 4;  // 16-position tiles that hold positions
  // rows [n, 16*nt) of V enter the last P.V tile with p = 0: make them zeros, not stale bits
  for (int i = t; i < (16 * nt - n) * 16; i += kAttnThreads)
    *reinterpret_cast<uint4*>(sV + (n + (i >> 4)) * kRowBytes + (i & 15) * 16) = make_uint4(0, 0, 0, 0);
  // q as the B operand of the scores, column gid = head (gid & 3), half (gid >> 2), all 128 dims
  uint32_t qb[8][2];
  {
    const float* qr = q + (size_t)b * ldq + (size_t)(kvh * kG + (gid & 3)) * kHD;
#pragma unroll
    for (int ks = 0; ks < 8; ks++) {
      const float2 x0 = *reinterpret_cast<const float2*>(qr + ks * 16 + tig * 2);
      const float2 x1 = *reinterpret_cast<const float2*>(qr + ks * 16 + 8 + tig * 2);
      qb[ks][0] = pack_hilo(x0.x, x0.y, gid >> 2);
      qb[ks][1] = pack_hilo(x1.x, x1.y, gid >> 2);
    }
  }
  asm volatile("cp.async.wait_group 1;" ::: "memory");  // all but the last group (V rows from row `old`)
  __syncthreads();

  // scores S[pos][col] = K[pos] . qcol: warp w takes positions 16w .. 16w+15; after adding the
  // lo column to the hi one (lane ^ 2), lanes with tig&1 == j hold heads 2j, 2j+1 for
  // positions 16w+gid (s[0][.]) and 16w+gid+8 (s[1][.])
  const int hb = (tig & 1) * 2;
  float s_[2][2];
  {
    float cacc[4] = {0.f, 0.f, 0.f, 0.f};
    if (warp < nt) {
      const uint8_t* arow = sK + (warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * kRowBytes + (lane >> 4) * 16;
#pragma unroll
      for (int ks = 0; ks < 8; ks++) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(arow + ks * 32, a0, a1, a2, a3);
        mma_bf16_16816(cacc, a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) cacc[i] += __shfl_xor_sync(0xffffffffu, cacc[i], 2);
    const int p0 = warp * 16 + gid, p1 = p0 + 8;
    s_[0][0] = p0 < n ? cacc[0] * scale : -INFINITY;
    s_[0][1] = p0 < n ? cacc[1] * scale : -INFINITY;
    s_[1][0] = p1 < n ? cacc[2] * scale : -INFINITY;
    s_[1][1] = p1 < n ? cacc[3] * scale : -INFINITY;
  }
  // per-head max and sum: rows, then the 8 gid lanes, then the 8 warps in order
#pragma unroll
  for (int j = 0; j < 2; j++) {
    float m = fmaxf(s_[0][j], s_[1][j]);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane < 2) red_max[(hb + j) * 8 + warp] = m;
  }
  __syncthreads();
  float Mh[2];
#pragma unroll
  for (int j = 0; j < 2; j++) {
    float m = red_max[(hb + j) * 8];
#pragma unroll
    for (int w = 1; w < 8; w++) m = fmaxf(m, red_max[(hb + j) * 8 + w]);
    Mh[j] = m;
  }
#pragma unroll
  for (int j = 0; j < 2; j++) {
    const float e0 = expf(s_[0][j] - Mh[j]), e1 = expf(s_[1][j] - Mh[j]);  // exp(-inf) = 0
    float sm = e0 + e1;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
    if (lane < 2) red_sum[(hb + j) * 8 + warp] = sm;
    if (tig < 2 && warp < nt) {  // P operand rows: hi of head h at row h, lo at row h + 4
      const int p0 = warp * 16 + gid;
      const uint16_t h0 = f2bf_bits(e0), h1 = f2bf_bits(e1);
      phl[(hb + j) * kPhlLd + p0] = h0;
      phl[(hb + j) * kPhlLd + p0 + 8] = h1;
      phl[(hb + j + 4) * kPhlLd + p0] = f2bf_bits(e0 - bf2f(h0));
      phl[(hb + j + 4) * kPhlLd + p0 + 8] = f2bf_bits(e1 - bf2f(h1));
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");  // the V rows
  __syncthreads();
  if constexpr (FUSED) grid_dep_launch();
  // P.V: O^T[d][col] = V^T[d] . P[col]; warp w takes dims 16w .. 16w+15 over the nt tiles
  {
    float cacc[4] = {0.f, 0.f, 0.f, 0.f};
    const uint8_t* vrow = sV + ((lane & 7) + (lane >> 4) * 8) * kRowBytes + warp * 32 + ((lane >> 3) & 1) * 16;
    const uint16_t* prow = phl + gid * kPhlLd + tig * 2;
    for (int ks = 0; ks < nt; ks++) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4_t(vrow + ks * 16 * kRowBytes, a0, a1, a2, a3);
      const uint32_t b0 = *reinterpret_cast<const uint32_t*>(prow + ks * 16);
      const uint32_t b1 = *reinterpret_cast<const uint32_t*>(prow + ks * 16 + 8);
      mma_bf16_16816(cacc, a0, a1, a2, a3, b0, b1);
    }
#pragma unroll
    for (int i = 0; i < 4; i++) cacc[i] += __shfl_xor_sync(0xffffffffu, cacc[i], 2);
    if (tig < 2) {
      const int d0 = warp * 16 + gid;
      ored[hb * kHD + d0] = cacc[0];
      ored[(hb + 1) * kHD + d0] = cacc[1];
      ored[hb * kHD + d0 + 8] = cacc[2];
      ored[(hb + 1) * kHD + d0 + 8] = cacc[3];
    }
  }
  __syncthreads();
  float acc[2], lsum[2], mx[2];
#pragma unroll
  for (int gg = 0; gg < 2; gg++) {
    const int g = 2 * hp + gg;
    acc[gg] = ored[g * kHD + tt];
    float m = red_max[g * 8], l = red_sum[g * 8];
#pragma unroll
    for (int w = 1; w < 8; w++) {
      m = fmaxf(m, red_max[g * 8 + w]);
      l += red_sum[g * 8 + w];
    }
    mx[gg] = m;
    lsum[gg] = l;
  }
  if constexpr (!FUSED) {
#pragma unroll
    for (int gg = 0; gg < 2; gg++) {
      float* rec = rec0 + (size_t)(2 * hp + gg) * nchunk * PS;
      rec[tt] = acc[gg];
      if (tt == 0) {
        rec[kHD] = mx[gg];
        rec[kHD + 1] = lsum[gg];
      }
    }
  } else {
    const uint32_t flag = (uint32_t)epoch + 1u;
    // records of this (stream, kv head): [chunk][g][PS] words
    unsigned long long* grp = recw + ((size_t)b * NKV + kvh) * nchunk * kG * PS;
    if (c > 0) {
      unsigned long long* rc = grp + (size_t)c * kG * PS;
#pragma unroll
      for (int gg = 0; gg < 2; gg++) {
        unsigned long long* rg = rc + (2 * hp + gg) * PS;
        st_rec(rg + tt, acc[gg], flag);
        if (tt == 0) {
          st_rec(rg + kHD, mx[gg], flag);
          st_rec(rg + kHD + 1, lsum[gg], flag);
        }
      }
      return;
    }
    // chunk 0: the combine needs the max of m over all chunks before the weighted sums, so it
    // polls the records of chunks 1..nc-1 (kRecChunks per round) for the max, then adds them
    // in chunk order from the words already read (re-read in batches for longer caches)
    const int nc = (P + kChunk - 1) / kChunk;
    float M[2], L[2], O[2];
#pragma unroll
    for (int gg = 0; gg < 2; gg++) M[gg] = fmaxf(-INFINITY, mx[gg]);
    unsigned long long w[kRecChunks][2][3];
    auto load_batch = [&](int c0, uint32_t mask) {
#pragma unroll
      for (int k = 0; k < kRecChunks; k++) {
        if (mask & (1u << k)) {
          const unsigned long long* rc = grp + (size_t)(c0 + k) * kG * PS;
#pragma unroll
          for (int gg = 0; gg < 2; gg++) {
            const unsigned long long* rg = rc + (2 * hp + gg) * PS;
            w[k][gg][0] = ld_rec(rg + tt);
            w[k][gg][1] = ld_rec(rg + kHD);
            w[k][gg][2] = ld_rec(rg + kHD + 1);
          }
        }
      }
    };
    bool ok = true;
    for (int c0 = 1; c0 < nc; c0 += kRecChunks) {  // pass 1: wait (bounded) and take the max
      uint32_t pend = 0;
#pragma unroll
      for (int k = 0; k < kRecChunks; k++)
        if (c0 + k < nc) pend |= 1u << k;
      load_batch(c0, pend);
      uint64_t t0 = 0;
      while (true) {
#pragma unroll
        for (int k = 0; k < kRecChunks; k++) {
          if (pend & (1u << k)) {
            bool ready = true;
#pragma unroll
            for (int gg = 0; gg < 2; gg++)
#pragma unroll
              for (int e = 0; e < 3; e++) ready &= (uint32_t)(w[k][gg][e] >> 32) == flag;
            if (ready) pend &= ~(1u << k);
          }
        }
        if (pend == 0 || !ok) break;
        const uint64_t now = globaltimer();
        if (t0 == 0) {
          t0 = now;
        } else if (now - t0 > kWaitTimeoutNs) {
          atomicCAS(&g_status_attn, 0, ST_ATTN_WAIT);
          ok = false;
          break;
        }
        load_batch(c0, pend);
      }
#pragma unroll
      for (int k = 0; k < kRecChunks; k++)
        if (c0 + k < nc)
#pragma unroll
          for (int gg = 0; gg < 2; gg++) M[gg] = fmaxf(M[gg], __uint_as_float((uint32_t)w[k][gg][1]));
    }
    // pass 2: exp-weighted sums in chunk order, chunk 0 from registers
#pragma unroll
    for (int gg = 0; gg < 2; gg++) {
      const float f = expf(mx[gg] - M[gg]);
      L[gg] = fmaf(lsum[gg], f, 0.f);
      O[gg] = fmaf(acc[gg], f, 0.f);
    }
    for (int c0 = 1; c0 < nc; c0 += kRecChunks) {
      uint32_t have = 0;
#pragma unroll
      for (int k = 0; k < kRecChunks; k++)
        if (c0 + k < nc) have |= 1u << k;
      if (nc > 1 + kRecChunks) load_batch(c0, have);  // else w still holds this (only) batch
#pragma unroll
      for (int k = 0; k < kRecChunks; k++) {
        if (have & (1u << k)) {
#pragma unroll
          for (int gg = 0; gg < 2; gg++) {
            const float m = __uint_as_float((uint32_t)w[k][gg][1]);
            if (m == -INFINITY) continue;
            const float f = expf(m - M[gg]);
            L[gg] = fmaf(__uint_as_float((uint32_t)w[k][gg][2]), f, L[gg]);
            O[gg] = fmaf(__uint_as_float((uint32_t)w[k][gg][0]), f, O[gg]);
          }
        }
      }
    }
#pragma unroll
    for (int gg = 0; gg < 2; gg++) {
      const float ov = O[gg] / L[gg];
      const size_t col = (size_t)(kvh * kG + 2 * hp + gg) * kHD + tt;
      const uint16_t hi = f2bf_bits(ov);
      act[(size_t)b * ld_act + col] = hi;
      act[(size_t)(16 + b) * ld_act + col] = f2bf_bits(ov - bf2f(hi));
    }
    if (t == 0) epochs[(size_t)b * NKV + kvh] = epoch + 1;  // read by the next launch only
  }
}

__global__ void __launch_bounds__(kAttnThreads) attn_partial_kernel(const float* __restrict__ q, int ldq,
                                                           const uint16_t* __restrict__ kc,
                                                           const uint16_t* __restrict__ vc,
                                                           const int32_t* __restrict__ pos, int NH,
                                                           int NKV, int S, float* __restrict__ part) {
  attn_chunk<false>(q, ldq, kc, vc, pos, nullptr, NH, NKV, S, part, nullptr, nullptr, nullptr, 0);
}

__global__ void __launch_bounds__(kAttnThreads, 3) attn_fused_kernel(const float* __restrict__ q, int ldq,
                                                         const uint16_t* __restrict__ kc,
                                                         const uint16_t* __restrict__ vc,
                                                         const int32_t* __restrict__ pos,
                                                         const int32_t* __restrict__ lanes, int NH, int NKV,
                                                         int S, unsigned long long* __restrict__ recw,
                                                         int* __restrict__ epochs, uint16_t* __restrict__ act,
                                                         int ld_act) {
  attn_chunk<true>(q, ldq, kc, vc, pos, lanes, NH, NKV, S, nullptr, recw, epochs, act, ld_act);
}

// Combines the chunk partials of one (stream, head) in chunk order.
// grid (NH, B), block HD.
__global__ void attn_combine_kernel(const float* __restrict__ part, int nchunk, float* __restrict__ ao,
                                    int ldao, int NH, uint16_t* __restrict__ act, int ld_act) {
  grid_dep_wait();
  grid_dep_launch();
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const int PS = kHD + 2;
  const float* rec = part + ((size_t)b * NH + h) * nchunk * PS;
  float M = -INFINITY;
  for (int c = 0; c < nchunk; c++) M = fmaxf(M, rec[(size_t)c * PS + kHD]);
  float L = 0.f, O = 0.f;
  for (int c = 0; c < nchunk; c++) {
    const float m = rec[(size_t)c * PS + kHD];
    if (m == -INFINITY) continue;
    const float f = expf(m - M);
    L = fmaf(rec[(size_t)c * PS + kHD + 1], f, L);
    O = fmaf(rec[(size_t)c * PS + d], f, O);
  }
  const float o = O / L;
  const size_t col = (size_t)h * kHD + d;
  if (act != nullptr) {  // hi/lo bf16 operand of the O-projection GEMM
    const uint16_t hi = f2bf_bits(o);
    act[(size_t)b * ld_act + col] = hi;
    act[(size_t)(16 + b) * ld_act + col] = f2bf_bits(o - bf2f(hi));
  } else {
    ao[(size_t)b * ldao + col] = o;
  }
}

static int launch_attn(const float* q, int ldq, const void* kc, const void* vc, const int32_t* pos, int B, int NH,
                       int NKV, int HD, int S, float* part, float* ao, int ldao, uint16_t* act, int ld_act,
                       cudaStream_t s) {
  RNGD_REQUIRE(q && kc && vc && pos && part && (ao || act), "attn_decode: null pointer");
  RNGD_REQUIRE(HD == kHD && NH == kG * NKV, "attn_decode: built for HD=128 and 4 query heads per kv head");
  RNGD_REQUIRE(S % kChunk == 0 && S > 0 && S <= 8192, "attn_decode: S=%d must be a multiple of 128", S);
  RNGD_REQUIRE(B >= 1, "attn_decode: B=%d", B);
  const int nchunk = S / kChunk;
  static std::atomic<unsigned long long> smem_set{0};
  RNGD_TRY(set_smem_limit_once((const void*)attn_partial_kernel, (int)kAttnSmem, &smem_set,
                               "cudaFuncSetAttribute(attn_partial_kernel)"));
  RNGD_TRY(launch_pdl(attn_partial_kernel, dim3(nchunk, NKV, B), dim3(kAttnThreads), kAttnSmem, s, "attn_partial_kernel", q, ldq,
                      (const uint16_t*)kc, (const uint16_t*)vc, pos, NH, NKV, S, part));
  return launch_pdl(attn_combine_kernel, dim3(NH, B), dim3(kHD), 0, s, "attn_combine_kernel", (const float*)part,
                    nchunk, ao, ldao, NH, act, ld_act);
}

int launch_attn_decode(const float* q, int ldq, const void* kc, const void* vc, const int32_t* pos, int B, int NH,
                       int NKV, int HD, int S, float* part, float* ao, int ldao, cudaStream_t s) {
  return launch_attn(q, ldq, kc, vc, pos, B, NH, NKV, HD, S, part, ao, ldao, nullptr, 0, s);
}

// Fused-attention scratch of the decode step (4-byte units): [16][NKV] int32 epochs (padded to
// 16 bytes), then [B][NKV][S/128][4][HD+2] 64-bit record words.  Zeroed once.
static size_t attn_epoch_units(int NKV) { return ((size_t)16 * NKV + 3) / 4 * 4; }

size_t attn_fused_scratch_units(int Bcap, int NKV, int S) {
  return attn_epoch_units(NKV) + 2 * (size_t)Bcap * NKV * (S / kChunk) * kG * (kHD + 2);
}

// The decode step's attention: one fused grid (chunks, combine, hi/lo operand of the O GEMM).
int launch_attn_decode_act(const float* q, int ldq, const void* kc, const void* vc, const int32_t* pos,
                           const int32_t* lanes, int B, int NH, int NKV, int HD, int S, float* part, void* act,
                           int ld_act, cudaStream_t s) {
  RNGD_REQUIRE(q && kc && vc && pos && part && act, "attn_decode: null pointer");
  RNGD_REQUIRE(HD == kHD && NH == kG * NKV, "attn_decode: built for HD=128 and 4 query heads per kv head");
  RNGD_REQUIRE(S % kChunk == 0 && S > 0 && S <= 8192, "attn_decode: S=%d must be a multiple of 128", S);
  RNGD_REQUIRE(B >= 1 && B <= 16, "attn_decode: B=%d outside 1..16", B);
  const int nchunk = S / kChunk;
  static std::atomic<unsigned long long> smem_set{0};
  RNGD_TRY(set_smem_limit_once((const void*)attn_fused_kernel, (int)kAttnSmem, &smem_set,
                               "cudaFuncSetAttribute(attn_fused_kernel)"));
  int* epochs = (int*)part;
  unsigned long long* recw = (unsigned long long*)(part + attn_epoch_units(NKV));
  return launch_pdl(attn_fused_kernel, dim3(nchunk, NKV, B), dim3(kAttnThreads), kAttnSmem, s, "attn_fused_kernel", q, ldq,
                    (const uint16_t*)kc, (const uint16_t*)vc, pos, lanes, NH, NKV, S, recw, epochs, (uint16_t*)act,
                    ld_act);
}

int read_status_attn(int* st, int reset) {
  RNGD_TRY(check_cuda(cudaMemcpyFromSymbol(st, g_status_attn, sizeof(int)), "read device status"));
  if (reset) {
    const int zero = 0;
    RNGD_TRY(check_cuda(cudaMemcpyToSymbol(g_status_attn, &zero, sizeof(int)), "reset device status"));
  }
  return RNGD_OK;
}

// ----------------------------------------------------------- SwiGLU
// act[b][f] = silu(g) * u with g, u from the 64-row interleaved gate/up output
// (kernels/decode_batch.py:159-161: g / (1 + exp(-g)) * u).
__global__ void swiglu_kernel(const float* __restrict__ gu, int ldgu, int Mi, float* __restrict__ act,
                              int ldact) {
  const int b = blockIdx.y;
  for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < Mi; f += gridDim.x * blockDim.x) {
    const int blk = f >> 6, j = f & 63;
    const float g = gu[(size_t)b * ldgu + blk * 128 + j];
    const float u = gu[(size_t)b * ldgu + blk * 128 + 64 + j];
    act[(size_t)b * ldact + f] = g / (1.0f + expf(-g)) * u;
  }
}

// ------------------------------------------------------------ embedding
__global__ void embed_kernel(const uint16_t* __restrict__ emb, const int32_t* __restrict__ toks, int H,
                             int V, float* __restrict__ x) {
  grid_dep_wait();
  grid_dep_launch();
  const int b = blockIdx.x;
  int t = toks[b];
  t = t < 0 ? 0 : (t >= V ? V - 1 : t);
  const uint16_t* row = emb + (size_t)t * H;
  for (int k = threadIdx.x; k < H; k += blockDim.x) x[(size_t)b * H + k] = bf2f(row[k]);
}

// --------------------------------------------------------------- argmax
// First maximum of each row (torch.argmax / numpy argmax tie rule,
// engines/decode_batch.py:162-171).  One CTA per row.
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ logits, int V,
                                                      int32_t* __restrict__ out) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  const float* row = logits + (size_t)blockIdx.x * V;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = row[i];
    if (v > best) { best = v; idx = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
  }
  if ((threadIdx.x & 31) == 0) { bv[threadIdx.x >> 5] = best; bi[threadIdx.x >> 5] = idx; }
  __syncthreads();
  if (threadIdx.x < 32) {
    best = bv[threadIdx.x];
    idx = bi[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
    }
    if (threadIdx.x == 0) out[blockIdx.x] = idx;
  }
}

__global__ void advance_kernel(int32_t* __restrict__ toks, int32_t* __restrict__ pos,
                               const int32_t* __restrict__ next, int B) {
  const int b = threadIdx.x;
  if (b < B) {
    toks[b] = next[b];
    pos[b] += 1;
  }
}

// ------------------------------------------------ allocation-free attention
// Library-owned scratch for rngd_attn_decode_noalloc: room for 4096 chunk
// partial records of HD + 2 floats (B * NH * S/128 <= 4096, e.g. 16 streams x
// 32 heads x S <= 1024), 2,129,920 bytes.  Every GPU that loads the library
// holds it until the process exits.
constexpr int kNoAllocRecords = 4096;
static __device__ __align__(256) float g_attn_scratch[kNoAllocRecords * (kHD + 2)];

// Device address of g_attn_scratch, looked up once per device with that device
// current (in host code the symbol itself is only a host-side stand-in).
static std::mutex g_scratch_mu;
static float* g_scratch_ptr[128] = {};

static int noalloc_scratch(float** out) {
  int dev = 0;
  RNGD_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  RNGD_REQUIRE(dev >= 0 && dev < 128, "attn_decode_noalloc: device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> g(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    RNGD_TRY(check_cuda(cudaGetSymbolAddress(&p, g_attn_scratch), "cudaGetSymbolAddress(attention scratch)"));
    g_scratch_ptr[dev] = (float*)p;
  }
  *out = g_scratch_ptr[dev];
  return RNGD_OK;
}

int launch_embed(const void* emb, const int32_t* toks, int H, int V, float* x, int B, cudaStream_t s) {
  return launch_pdl(embed_kernel, dim3(B), dim3(256), 0, s, "embed_kernel", (const uint16_t*)emb, toks, H, V, x);
}

}  // namespace rngd

using namespace rngd;

extern "C" int rngd_gemv_bf16(const void* W, int N, int K, const float* X, int ldx, int B, float* Y, int ldy,
                              int accumulate, rngd_stream_t stream) {
  return launch_gemv(W, N, K, X, ldx, B, Y, ldy, accumulate, (cudaStream_t)stream);
}

extern "C" int rngd_rmsnorm_f32(const float* x, int R, int H, const float* w, float eps, float* out,
                                rngd_stream_t stream) {
  return launch_rmsnorm(x, R, H, w, eps, out, (cudaStream_t)stream);
}

extern "C" int rngd_attn_decode(const float* q, const void* kc, const void* vc, const int32_t* pos, int B,
                                int Bcap, int NH, int NKV, int HD, int S, float* part, float* ao,
                                rngd_stream_t stream) {
  RNGD_REQUIRE(B <= Bcap, "attn_decode: B=%d > Bcap=%d", B, Bcap);
  return launch_attn_decode(q, NH * HD, kc, vc, pos, B, NH, NKV, HD, S, part, ao, NH * HD,
                            (cudaStream_t)stream);
}

extern "C" int rngd_attn_decode_noalloc(const float* q, const void* kc, const void* vc, const int32_t* pos,
                                        int B, int Bcap, int NH, int NKV, int HD, int S, float* ao,
                                        rngd_stream_t stream) {
  RNGD_REQUIRE(B >= 1 && B <= Bcap, "attn_decode_noalloc: B=%d outside 1..Bcap=%d", B, Bcap);
  RNGD_REQUIRE(HD == kHD && NH == kG * NKV, "attn_decode_noalloc: built for HD=128 and 4 query heads per kv head");
  RNGD_REQUIRE(S % kChunk == 0 && S > 0, "attn_decode_noalloc: S=%d must be a positive multiple of 128", S);
  const long records = (long)B * NH * (S / kChunk);
  RNGD_REQUIRE(records <= kNoAllocRecords,
               "attn_decode_noalloc: B*NH*S/128 = %ld partial records exceed the built-in scratch of %d "
               "(e.g. B=16, NH=32 allows S <= 1024); use rngd_attn_decode with caller-owned scratch",
               records, kNoAllocRecords);
  float* part = nullptr;
  RNGD_TRY(noalloc_scratch(&part));
  return launch_attn(q, NH * HD, kc, vc, pos, B, NH, NKV, HD, S, part, ao, NH * HD, nullptr, 0,
                     (cudaStream_t)stream);
}

extern "C" int rngd_decode_advance(const rngd_decode_io_t* io, rngd_stream_t stream) {
  RNGD_REQUIRE(io && io->toks && io->pos && io->next && io->B >= 1 && io->B <= 1024, "advance: bad io");
  advance_kernel<<<1, 32 * ((io->B + 31) / 32), 0, (cudaStream_t)stream>>>((int32_t*)io->toks, (int32_t*)io->pos,
                                                                          io->next, io->B);
  return check_launch("advance_kernel");
}
