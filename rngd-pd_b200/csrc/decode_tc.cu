// Tensor-core decode step: weight-streaming tcgen05 GEMMs with fused epilogues.
//
// A decode GEMM is Y[b][n] = sum_k W[n][k] * h[b][k] with W bf16 (HBM, read
// once per step) and h fp32.  It runs on tcgen05 as D = A * B^T with
//   A = a 128-row tile of W (TMA, 128-byte swizzle, K-major),
//   B = the activation operand: 32 bf16 rows = 16 streams x {hi, lo}, where
//       hi = bf16(h) and lo = bf16(h - hi), so hi + lo carries ~16 mantissa
//       bits of the fp32 activation and W*hi + W*lo (fp32 accumulation in
//       TMEM) stays at fp32-level accuracy,
//   D = 128 x 32 fp32 accumulators in tensor memory.
// Work unit = (128-row tile, K split).  Split decisions depend only on the
// matrix shape (never on B), and the last CTA to finish a tile sums the split
// partials in split order, so every stream's result is deterministic and
// independent of which other streams share the batch.
//
// Epilogues (run by the CTA that completes a tile):
//   QKV     RoPE (rotate-half, fp32 angles) on q and k; q -> fp32 buffer,
//           k and v -> bf16 cache at pos[b]      (kernels/decode_batch.py:77-82)
//   RESID   x[b][n] += y                          (zipadd, kernels/decode_batch.py:87,91)
//   SWIGLU  silu(gate) * up for the tile's 64 features -> hi/lo operand of the
//           down GEMM                             (kernels/decode_batch.py:88-90)
//   LOGITS  logits[b][n] = y and a first-max argmax key per stream
//                                                 (engines/decode_batch.py:122-171)
#include <mutex>
#include <unordered_map>

#include "tc.cuh"

namespace rngd {

__device__ int g_status_decode = 0;  // this file's bounded-wait status word

constexpr int BM = 128, BK = 64, BNC = 32, MAXB = 16;
constexpr int A_BYTES = BM * BK * 2;   // 16 KB weight tile per stage
constexpr int B_BYTES = BNC * BK * 2;  // 4 KB activation tile per stage
constexpr int STAGES = 4;
constexpr int YS_LD = 17;

enum Epi : int { EPI_QKV = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_LOGITS = 3 };

struct GemmArgs {
  int N, K, nkb, nsplit, layer, B;
  float* partial;
  int* counters;
  // QKV
  const int32_t* pos;
  const float* inv;
  float* q;
  int ldq;
  uint16_t* kc;
  uint16_t* vc;
  int NH, NKV, S;
  // RESID
  float* x;
  int ldx;
  // SWIGLU
  uint16_t* act_out;
  int ld_act;
  // LOGITS
  float* logits;
  unsigned long long* best;
  int V;
};

constexpr size_t kSmemBytes = 1024 /*align*/ + STAGES * (A_BYTES + B_BYTES) + 3 * STAGES * 8 + 64 +
                              BM * YS_LD * 4 + 64;

__device__ __forceinline__ uint32_t orderable(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <int EPI>
__global__ void __launch_bounds__(128) wsgemm_kernel(const __grid_constant__ CUtensorMap tmW,
                                                     const __grid_constant__ CUtensorMap tmX, GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = base;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint64_t* full = (uint64_t*)(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* accum = empty + STAGES;
  uint32_t* tmem_slot = (uint32_t*)(accum + 1);
  int* s_last = (int*)(tmem_slot + 1);
  float* ys = (float*)(base + STAGES * (A_BYTES + B_BYTES) + 3 * STAGES * 8 + 64);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int unit = blockIdx.x;
  const int tile = unit / a.nsplit, split = unit - tile * a.nsplit;
  const int kb0 = (int)((long)split * a.nkb / a.nsplit), kb1 = (int)((long)(split + 1) * a.nkb / a.nsplit);
  const int nk = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // TMA producer: weight tile + activation tile per 64-wide K block
    for (int i = 0; i < nk; i++) {
      const int s = i % STAGES;
      const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
      if (!mbar_wait(&empty[s], ph ^ 1u, ST_TMA_WAIT, &g_status_decode)) break;
      mbar_arrive_expect_tx(&full[s], A_BYTES + B_BYTES);
      const int k = (kb0 + i) * BK;
      tma_load_3d(sA + s * A_BYTES, &tmW, &full[s], k, tile * BM, a.layer);
      tma_load_2d(sB + s * B_BYTES, &tmX, &full[s], k, 0);
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer: 4 x (128x32x16) per stage, accumulating in TMEM
    const uint32_t idesc = idesc_bf16_f32(BM, BNC);
    bool ok = true;
    for (int i = 0; i < nk && ok; i++) {
      const int s = i % STAGES;
      const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
      ok = mbar_wait(&full[s], ph, ST_MMA_WAIT, &g_status_decode);
      if (!ok) break;
      tc_fence_after();
      const uint32_t aBase = smem_u32(sA + s * A_BYTES), bBase = smem_u32(sB + s * B_BYTES);
#pragma unroll
      for (int kk = 0; kk < BK / 16; kk++)
        umma_bf16(tmem, sw128_kmajor_desc(aBase + kk * 32), sw128_kmajor_desc(bBase + kk * 32), idesc,
                  (i | kk) != 0);
      umma_commit(&empty[s]);
    }
    umma_commit(accum);
  }
  __syncwarp();

  // ---- accumulators -> registers (thread r owns row r of the tile)
  mbar_wait(accum, 0, ST_EPI_WAIT, &g_status_decode);
  tc_fence_after();
  float v[32];
  tmem_ld_32x32b_x32(tmem + ((uint32_t)(warp * 32) << 16), v);
  tc_fence_before();
  __syncthreads();
  if (warp == 2) tmem_dealloc(tmem, 32);

  const int r = threadIdx.x;
  const int n = tile * BM + r;
  float y[MAXB];
#pragma unroll
  for (int b = 0; b < MAXB; b++) y[b] = v[b] + v[MAXB + b];

  if (a.nsplit > 1) {
    float4* dst = reinterpret_cast<float4*>(a.partial + ((size_t)split * a.N + n) * MAXB);
#pragma unroll
    for (int j = 0; j < 4; j++) __stcg(dst + j, make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]));
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *s_last = (atomicAdd(&a.counters[tile], 1) == a.nsplit - 1);
    __syncthreads();
    if (!*s_last) return;
    __threadfence();
#pragma unroll
    for (int b = 0; b < MAXB; b++) y[b] = 0.f;
    for (int s = 0; s < a.nsplit; s++) {
      const float4* src = reinterpret_cast<const float4*>(a.partial + ((size_t)s * a.N + n) * MAXB);
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float4 t = __ldcg(src + j);
        y[4 * j] += t.x; y[4 * j + 1] += t.y; y[4 * j + 2] += t.z; y[4 * j + 3] += t.w;
      }
    }
    if (threadIdx.x == 0) a.counters[tile] = 0;  // ready for the next launch
  }

  if constexpr (EPI == EPI_RESID) {
    for (int b = 0; b < a.B; b++) a.x[(size_t)b * a.ldx + n] += y[b];
  } else if constexpr (EPI == EPI_QKV) {
#pragma unroll
    for (int b = 0; b < MAXB; b++) ys[r * YS_LD + b] = y[b];
    __syncthreads();
    const int head = tile;  // one 128-row tile = one head
    const int i = r & 63;
    const bool lo_half = r < 64;
    const int partner = r ^ 64;
    if (head < a.NH + a.NKV) {
      for (int b = 0; b < a.B; b++) {
        const int p = a.pos[b];
        float sn, cs;
        sincosf((float)p * a.inv[i], &sn, &cs);
        const float other = ys[partner * YS_LD + b];
        const float o = lo_half ? y[b] * cs - other * sn : y[b] * cs + other * sn;
        if (head < a.NH) {
          a.q[(size_t)b * a.ldq + n] = o;
        } else if (p >= 0 && p < a.S) {
          a.kc[(((size_t)b * a.NKV + (head - a.NH)) * a.S + p) * 128 + r] = f2bf_bits(o);
        }
      }
    } else {
      for (int b = 0; b < a.B; b++) {
        const int p = a.pos[b];
        if (p >= 0 && p < a.S)
          a.vc[(((size_t)b * a.NKV + (head - a.NH - a.NKV)) * a.S + p) * 128 + r] = f2bf_bits(y[b]);
      }
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll
    for (int b = 0; b < MAXB; b++) ys[r * YS_LD + b] = y[b];
    __syncthreads();
    if (r < 64) {
      const int f = tile * 64 + r;
      for (int b = 0; b < a.B; b++) {
        const float g = y[b], u = ys[(r + 64) * YS_LD + b];
        const float act = g / (1.0f + expf(-g)) * u;
        const uint16_t hi = f2bf_bits(act);
        a.act_out[(size_t)b * a.ld_act + f] = hi;
        a.act_out[(size_t)(MAXB + b) * a.ld_act + f] = f2bf_bits(act - bf2f(hi));
      }
    }
  } else if constexpr (EPI == EPI_LOGITS) {
    __shared__ unsigned long long red[4][MAXB];
    for (int b = 0; b < a.B; b++) {
      unsigned long long key = 0;
      if (n < a.V) {
        a.logits[(size_t)b * a.V + n] = y[b];
        key = ((unsigned long long)orderable(y[b]) << 32) | (0xFFFFFFFFu - (uint32_t)n);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, key, o);
        key = t > key ? t : key;
      }
      if (lane == 0) red[warp][b] = key;
    }
    __syncthreads();
    if (r < a.B) {
      unsigned long long k = red[0][r];
      for (int w = 1; w < 4; w++) k = red[w][r] > k ? red[w][r] : k;
      atomicMax(&a.best[r], k);
    }
  }
}

// ---------------------------------------------------------------- prep
// act[b] = bf16(h), act[16+b] = bf16(h - bf16(h)) with h = rms(x) * w (or
// h = x when w == nullptr).  Also clears the argmax keys when best != nullptr.
__global__ void __launch_bounds__(256) prep_act_kernel(const float* __restrict__ x, int ldx, int H,
                                                       const float* __restrict__ w, float eps,
                                                       uint16_t* __restrict__ act, int ld_act,
                                                       unsigned long long* best) {
  __shared__ float red[8];
  const int b = blockIdx.x;
  const float* xr = x + (size_t)b * ldx;
  float inv = 1.f;
  if (w != nullptr) {
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
    inv = red[0];
  }
  for (int k = threadIdx.x; k < H; k += 256) {
    const float h = w != nullptr ? xr[k] * inv * w[k] : xr[k];
    const uint16_t hi = f2bf_bits(h);
    act[(size_t)b * ld_act + k] = hi;
    act[(size_t)(MAXB + b) * ld_act + k] = f2bf_bits(h - bf2f(hi));
  }
  if (best != nullptr && threadIdx.x == 0) best[b] = 0ull;
}

__global__ void finalize_argmax_kernel(const unsigned long long* __restrict__ best, int32_t* __restrict__ next,
                                       int B) {
  const int b = threadIdx.x;
  if (b < B) next[b] = (int32_t)(0xFFFFFFFFu - (uint32_t)(best[b] & 0xFFFFFFFFull));
}

// ------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  });
  return fn;
}

int encode_tmap_bf16(CUtensorMap* out, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box) {
  EncodeTiledFn enc = get_encode();
  RNGD_REQUIRE(enc != nullptr, "cuTensorMapEncodeTiled is unavailable");
  RNGD_REQUIRE(((uintptr_t)base & 15) == 0, "tensor map base must be 16-byte aligned");
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; i++) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; i++) {
    RNGD_REQUIRE(strides_bytes[i] % 16 == 0, "tensor map strides must be multiples of 16 bytes");
    st[i] = strides_bytes[i];
  }
  CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void*>(base), d, st, bx, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return RNGD_ERR_CUDA;
  }
  return RNGD_OK;
}

// cached tensor maps: weights [L][N][K] (3-D) and activation operands [32][K] (2-D)
struct MapKey {
  const void* p;
  uint64_t a, b, c;
  bool operator==(const MapKey& o) const { return p == o.p && a == o.a && b == o.b && c == o.c; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.p) ^ (k.a * 0x9E3779B97F4A7C15ull) ^ (k.b << 21) ^ (k.c << 42);
  }
};
static std::mutex g_map_mu;
static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

static int weight_map(const void* w, int L, int N, int K, CUtensorMap* out) {
  MapKey key{w, (uint64_t)L, (uint64_t)N, (uint64_t)K};
  std::lock_guard<std::mutex> g(g_map_mu);
  auto it = g_maps.find(key);
  if (it != g_maps.end()) {
    *out = it->second;
    return RNGD_OK;
  }
  const uint64_t dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)L};
  const uint64_t strides[2] = {(uint64_t)K * 2, (uint64_t)K * 2 * N};
  const uint32_t box[3] = {BK, BM, 1};
  RNGD_TRY(encode_tmap_bf16(out, w, 3, dims, strides, box));
  g_maps[key] = *out;
  return RNGD_OK;
}

static int act_map(const void* act, int K, int ld, CUtensorMap* out) {
  MapKey key{act, (uint64_t)K, (uint64_t)ld, 0xAC7ull};
  std::lock_guard<std::mutex> g(g_map_mu);
  auto it = g_maps.find(key);
  if (it != g_maps.end()) {
    *out = it->second;
    return RNGD_OK;
  }
  const uint64_t dims[2] = {(uint64_t)K, (uint64_t)(2 * MAXB)};
  const uint64_t strides[1] = {(uint64_t)ld * 2};
  const uint32_t box[2] = {BK, BNC};
  RNGD_TRY(encode_tmap_bf16(out, act, 2, dims, strides, box));
  g_maps[key] = *out;
  return RNGD_OK;
}

// K splits per weight shape: about two waves of two CTAs per SM, at least
// 8 K blocks (128 KB of weights) per unit.  Depends on the shape only.
int decode_nsplit(int N, int K) {
  const int tiles = (N + BM - 1) / BM, nkb = K / BK;
  int s = (2 * 2 * kNumSMs + tiles - 1) / tiles;
  if (s > nkb / 8) s = nkb / 8;
  return s < 1 ? 1 : s;
}

template <int EPI>
static int launch_wsgemm(const void* W, int L, int layer, int N, int K, const void* act, int ld_act_in,
                         GemmArgs a, cudaStream_t s) {
  RNGD_REQUIRE(K % BK == 0 && K >= BK, "decode GEMM: K=%d must be a multiple of 64", K);
  RNGD_REQUIRE(N % BM == 0 || EPI == EPI_LOGITS, "decode GEMM: N=%d must be a multiple of 128", N);
  CUtensorMap tw, tx;
  RNGD_TRY(weight_map(W, L, N, K, &tw));
  RNGD_TRY(act_map(act, K, ld_act_in, &tx));
  a.N = N;
  a.K = K;
  a.nkb = K / BK;
  a.nsplit = EPI == EPI_LOGITS ? 1 : decode_nsplit(N, K);
  a.layer = layer;
  const int tiles = (N + BM - 1) / BM;
  static bool attr_set[4] = {false, false, false, false};
  if (!attr_set[EPI]) {
    RNGD_TRY(check_cuda(cudaFuncSetAttribute(wsgemm_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kSmemBytes),
                        "cudaFuncSetAttribute(wsgemm)"));
    attr_set[EPI] = true;
  }
  wsgemm_kernel<EPI><<<tiles * a.nsplit, 128, kSmemBytes, s>>>(tw, tx, a);
  return check_launch("wsgemm_kernel");
}

int launch_prep(const float* x, int ldx, int B, int H, const float* w, float eps, void* act, int ld_act,
                unsigned long long* best, cudaStream_t s) {
  prep_act_kernel<<<B, 256, 0, s>>>(x, ldx, H, w, eps, (uint16_t*)act, ld_act, best);
  return check_launch("prep_act_kernel");
}

int launch_attn_decode_act(const float* q, int ldq, const void* kc, const void* vc, const int32_t* pos, int B,
                           int NH, int NKV, int HD, int S, float* part, void* act, int ld_act, cudaStream_t s);

}  // namespace rngd

using namespace rngd;

static int check_tc_io(const rngd_model_t* m, const rngd_decode_io_t* io) {
  RNGD_REQUIRE(m && io, "null model or io");
  RNGD_REQUIRE(m->HD == 128 && m->NH == 4 * m->NKV, "decode: kernels are built for HD=128, NH=4*NKV");
  RNGD_REQUIRE(m->H % 128 == 0 && m->M % 64 == 0 && (2 * m->M) % 128 == 0 && m->H % 64 == 0,
               "decode: H and 2*M must be multiples of 128");
  RNGD_REQUIRE(io->B >= 1 && io->B <= 16 && io->B <= io->Bcap, "decode: B=%d outside 1..min(16, Bcap)", io->B);
  RNGD_REQUIRE(io->S % 128 == 0 && io->S > 0 && io->S <= 8192, "decode: S=%d must be a multiple of 128", io->S);
  RNGD_REQUIRE(io->kcache && io->vcache && io->toks && io->pos && io->x && io->q && io->act && io->act2 &&
                   io->logits && io->attn_part && io->partial && io->counters && io->best && io->next,
               "decode: null buffer");
  return RNGD_OK;
}

extern "C" int rngd_decode_workspace(const rngd_model_t* m, int S, size_t* partial_floats, size_t* counters,
                                     size_t* act_cols, size_t* act2_cols) {
  RNGD_REQUIRE(m && partial_floats && counters && act_cols && act2_cols, "workspace: null argument");
  const int QN = m->NH * m->HD, KN = m->NKV * m->HD;
  const int shapes[4][2] = {{QN + 2 * KN, m->H}, {m->H, QN}, {2 * m->M, m->H}, {m->H, m->M}};
  size_t pf = 0, ct = 0;
  for (auto& sh : shapes) {
    const int ns = decode_nsplit(sh[0], sh[1]);
    const size_t t = (size_t)(sh[0] + BM - 1) / BM;
    if (ns > 1) {
      pf = pf > (size_t)ns * sh[0] * MAXB ? pf : (size_t)ns * sh[0] * MAXB;
      ct = ct > t ? ct : t;
    }
  }
  *partial_floats = pf;
  *counters = ct;
  *act_cols = (size_t)(m->H > QN ? m->H : QN);
  *act2_cols = (size_t)m->M;
  (void)S;
  return RNGD_OK;
}

extern "C" int rngd_tc_gemv(const void* W, int N, int K, const float* X, int ldx, int B, float* Y, int ldy,
                            void* act, float* partial, int32_t* counters, rngd_stream_t stream) {
  RNGD_REQUIRE(W && X && Y && act, "tc_gemv: null pointer");
  RNGD_REQUIRE(B >= 1 && B <= MAXB, "tc_gemv: B=%d outside 1..16", B);
  RNGD_REQUIRE(N % BM == 0 && K % BK == 0, "tc_gemv: need N %% 128 == 0 and K %% 64 == 0 (N=%d K=%d)", N, K);
  RNGD_REQUIRE(decode_nsplit(N, K) == 1 || (partial && counters), "tc_gemv: split-K needs partial and counters");
  cudaStream_t s = (cudaStream_t)stream;
  RNGD_TRY(launch_prep(X, ldx, B, K, nullptr, 0.f, act, K, nullptr, s));
  GemmArgs a = {};
  a.B = B;
  a.partial = partial;
  a.counters = counters;
  a.x = Y;
  a.ldx = ldy;
  return launch_wsgemm<EPI_RESID>(W, 1, 0, N, K, act, K, a, s);
}

extern "C" int rngd_tc_gemv_workspace(int N, int K, size_t* partial_floats, size_t* counters) {
  RNGD_REQUIRE(partial_floats && counters, "tc_gemv_workspace: null argument");
  const int ns = decode_nsplit(N, K);
  *partial_floats = ns > 1 ? (size_t)ns * N * MAXB : 0;
  *counters = ns > 1 ? (size_t)(N / BM) : 0;
  return RNGD_OK;
}

extern "C" int rngd_decode_embed(const rngd_model_t* m, const rngd_decode_io_t* io, rngd_stream_t stream);

extern "C" int rngd_decode_layers(const rngd_model_t* m, const rngd_decode_io_t* io, int layer0, int layer1,
                                  rngd_stream_t stream) {
  RNGD_TRY(check_tc_io(m, io));
  RNGD_REQUIRE(0 <= layer0 && layer0 <= layer1 && layer1 <= m->L, "decode: layers [%d, %d) outside [0, %d)",
               layer0, layer1, m->L);
  RNGD_REQUIRE(layer1 - layer0 <= io->kv_layers, "decode: %d layers requested but the cache block holds %d",
               layer1 - layer0, io->kv_layers);
  cudaStream_t s = (cudaStream_t)stream;
  const int H = m->H, Mi = m->M, QN = m->NH * m->HD, KN = m->NKV * m->HD, NQKV = QN + 2 * KN;
  const int B = io->B;
  const int ld_act = H > QN ? H : QN;
  const size_t lane_elems = (size_t)m->NKV * io->S * m->HD;
  for (int l = layer0; l < layer1; l++) {
    uint16_t* kc = (uint16_t*)io->kcache + (size_t)(l - layer0) * io->Bcap * lane_elems;
    uint16_t* vc = (uint16_t*)io->vcache + (size_t)(l - layer0) * io->Bcap * lane_elems;
    GemmArgs a = {};
    a.B = B;
    a.partial = io->partial;
    a.counters = io->counters;
    // attention block
    RNGD_TRY(launch_prep(io->x, H, B, H, m->n1 + (size_t)l * H, m->eps, io->act, ld_act, nullptr, s));
    a.pos = io->pos; a.inv = m->inv_freq; a.q = io->q; a.ldq = QN; a.kc = kc; a.vc = vc;
    a.NH = m->NH; a.NKV = m->NKV; a.S = io->S;
    RNGD_TRY(launch_wsgemm<EPI_QKV>(m->wqkv, m->L, l, NQKV, H, io->act, ld_act, a, s));
    RNGD_TRY(launch_attn_decode_act(io->q, QN, kc, vc, io->pos, B, m->NH, m->NKV, m->HD, io->S, io->attn_part,
                                    io->act, ld_act, s));
    a.x = io->x; a.ldx = H;
    RNGD_TRY(launch_wsgemm<EPI_RESID>(m->wo, m->L, l, H, QN, io->act, ld_act, a, s));
    // MLP block
    RNGD_TRY(launch_prep(io->x, H, B, H, m->n2 + (size_t)l * H, m->eps, io->act, ld_act, nullptr, s));
    a.act_out = (uint16_t*)io->act2; a.ld_act = Mi;
    RNGD_TRY(launch_wsgemm<EPI_SWIGLU>(m->wgu, m->L, l, 2 * Mi, H, io->act, ld_act, a, s));
    RNGD_TRY(launch_wsgemm<EPI_RESID>(m->wd, m->L, l, H, Mi, io->act2, Mi, a, s));
  }
  return RNGD_OK;
}

extern "C" int rngd_decode_lmhead(const rngd_model_t* m, const rngd_decode_io_t* io, rngd_stream_t stream) {
  RNGD_TRY(check_tc_io(m, io));
  cudaStream_t s = (cudaStream_t)stream;
  const int H = m->H, QN = m->NH * m->HD;
  const int ld_act = H > QN ? H : QN;
  RNGD_TRY(launch_prep(io->x, H, io->B, H, m->norm, m->eps, io->act, ld_act, (unsigned long long*)io->best, s));
  GemmArgs a = {};
  a.B = io->B;
  a.logits = io->logits;
  a.best = (unsigned long long*)io->best;
  a.V = m->V;
  RNGD_TRY(launch_wsgemm<EPI_LOGITS>(m->lm, 1, 0, m->V, H, io->act, ld_act, a, s));
  finalize_argmax_kernel<<<1, 32, 0, s>>>((const unsigned long long*)io->best, io->next, io->B);
  return check_launch("finalize_argmax_kernel");
}

int rngd::read_status_decode(int* st, int reset) {
  RNGD_TRY(check_cuda(cudaMemcpyFromSymbol(st, g_status_decode, sizeof(int)), "read device status"));
  if (reset) {
    const int zero = 0;
    RNGD_TRY(check_cuda(cudaMemcpyToSymbol(g_status_decode, &zero, sizeof(int)), "reset device status"));
  }
  return RNGD_OK;
}

extern "C" int rngd_device_status(int* status, int reset) {
  RNGD_REQUIRE(status != nullptr, "device_status: null output");
  int st = 0;
  RNGD_TRY(read_status_decode(&st, reset));
  *status = st;
  return RNGD_OK;
}
