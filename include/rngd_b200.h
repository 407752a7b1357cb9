/* rngd_b200.h — C ABI of the B200 kernels behind rngd-pd's hot path.
 *
 * Plain pointers, sizes and a stream handle; no torch or Python types.  The
 * Python package rngd_pd (engines/, connector/, nvlink.py) binds these with
 * ctypes; a C/C++/Go/Rust host can bind them the same way.
 *
 * Every function returns an int status: RNGD_OK (0) or a negative code, and
 * records a message that rngd_last_error() copies out.  Device-side waits are
 * bounded and come back as RNGD_ERR_TIMEOUT; nothing traps.  All launches are
 * stream-ordered on the given stream (NULL = the legacy default stream).
 *
 * Reference interfaces each group replaces are cited per declaration
 * (paths relative to the rngd-pd repository).
 */
#ifndef RNGD_B200_H
#define RNGD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RNGD_OK 0
#define RNGD_ERR_ARG (-1)         /* bad argument: shape, pointer, bound */
#define RNGD_ERR_CUDA (-2)        /* a CUDA call or launch failed */
#define RNGD_ERR_TIMEOUT (-3)     /* a bounded device/host wait ran out */
#define RNGD_ERR_UNSUPPORTED (-4) /* a shape outside what the kernels are built for */

typedef void* rngd_stream_t; /* cudaStream_t */

/* ---------------------------------------------------------------- runtime */
/* Copies the last error message of the calling thread (NUL-terminated). */
int rngd_last_error(char* buf, size_t n);
/* ABI version of this library (bumped when a struct below changes). */
int rngd_abi_version(void);

/* ------------------------------------------------------- synthetic inputs
 * The reference serves a real checkpoint (src/rngd_pd/engines/decode_batch.py:
 * 456-462 loads it with transformers); this build measures on seeded synthetic
 * weights and KV instead.  Integer-only recipe, bit-identical to the CPU
 * generator of the test oracle: splitmix64 hash of (seed, tid, index), sum of
 * its four 16-bit fields (Irwin-Hall n=4) times `scale`, rounded to bf16. */
int rngd_synth_gauss_bf16(void* dst, uint64_t n, uint64_t seed, uint64_t tid, uint64_t start,
                          float scale, rngd_stream_t stream);
/* dst[i] = (hash(seed, tid, start+i) >> 32) % hi as int32 (token ids, lengths). */
int rngd_synth_uniform_i32(int32_t* dst, uint64_t n, uint64_t seed, uint64_t tid, uint64_t start,
                           uint32_t hi, rngd_stream_t stream);

/* ---------------------------------------------------------- model + decode
 * Weights as the engine lays them out in HBM (bf16, K-major rows, i.e. the HF
 * [out, in] layout), one contiguous block per kind over all layers. */
typedef struct rngd_model {
  int32_t H, M, NH, NKV, HD, L, V;
  float eps;
  const void* wqkv;      /* bf16 [L][(NH+2*NKV)*HD][H]: q rows, then k, then v */
  const void* wo;        /* bf16 [L][H][NH*HD] */
  const void* wgu;       /* bf16 [L][2*M][H]: gate/up interleaved in 64-row blocks */
  const void* wd;        /* bf16 [L][H][M] */
  const float* n1;       /* fp32 [L][H] input_layernorm */
  const float* n2;       /* fp32 [L][H] post_attention_layernorm */
  const float* norm;     /* fp32 [H] final norm */
  const void* embed;     /* bf16 [V][H] */
  const void* lm;        /* bf16 [V][H] */
  const float* inv_freq; /* fp32 [HD/2] RoPE inverse frequencies (device) */
} rngd_model_t;

/* Per-engine decode state.  Lanes 0..B-1 of the resident cache are the B
 * streams of the step; each has its own position (engines/decode_batch.py:422-442).
 * Activation operands of the tensor-core GEMMs are 32 bf16 rows: rows 0..15
 * hold bf16(h) of each stream, rows 16..31 bf16(h - bf16(h)); rows of streams
 * >= B stay zero (allocate zeroed). */
typedef struct rngd_decode_io {
  int32_t B;            /* streams stepped (<= 16) */
  int32_t Bcap;         /* lanes of the resident cache */
  int32_t S;            /* cache width in positions (multiple of 128, <= 8192) */
  int32_t kv_layers;    /* layers held by kcache/vcache (a layer group's block) */
  void* kcache;         /* bf16 [kv_layers][Bcap][NKV][S][HD], first layer = layer0 of the call */
  void* vcache;         /* bf16 [kv_layers][Bcap][NKV][S][HD] */
  const int32_t* toks;  /* device [B] token ids of this step */
  const int32_t* pos;   /* device [B] position each token is written at */
  float* x;             /* fp32 [16][H] residual stream */
  float* q;             /* fp32 [16][NH*HD] rotated queries */
  void* act;            /* bf16 [32][max(H, NH*HD)] operand of x * norm weight (zeroed at allocation) */
  void* act_o;          /* bf16 [32][NH*HD] attention-output operand (zeroed at allocation) */
  void* act2;           /* bf16 [32][M] down-projection operand (zeroed at allocation) */
  float* ss;            /* fp32 [H/128][16] per-128-column sums of squares of x (RMSNorm) */
  float* logits;        /* fp32 [B][V] */
  float* attn_part;     /* attention scratch, rngd_decode_attn_workspace() 4-byte units, zeroed once */
  float* partial;       /* split-tile scratch, rngd_decode_workspace() 4-byte units (16-byte aligned),
                           zeroed once */
  int32_t* counters;    /* split-tile epochs, rngd_decode_workspace() int32 entries, zeroed once */
  uint64_t* best;       /* [16] argmax keys */
  int32_t* next;        /* device [B] greedy next tokens */
  const int32_t* lanes; /* optional device [B]: the cache lane of each stream (< Bcap); NULL = stream b
                           uses lane b.  Streams may share a lane at distinct positions: a chunk of
                           one sequence's prompt (engines/prefill_chunk.py:109-142), where stream c
                           holds position base + c and attends to the lane's positions <= its own. */
} rngd_decode_io_t;

/* Sizes of the decode scratch buffers for a model (shape-only; independent of B). */
int rngd_decode_workspace(const rngd_model_t* m, int S, size_t* partial_floats, size_t* counters,
                          size_t* act_cols, size_t* act2_cols);
/* Size of io->attn_part for streams 0..Bcap-1 (Bcap <= 16) of S cache positions: chunk
 * records of the fused decode attention plus an epoch per (stream, kv head). */
int rngd_decode_attn_workspace(const rngd_model_t* m, int Bcap, int S, size_t* attn_units);
/* Device status word of the bounded waits (0 = none timed out); reset clears it. */
int rngd_device_status(int* status, int reset);

/* x = embed[toks] (engines/decode_batch.py:432), plus the first layer's
 * operand x * n1[0] and its sums of squares; clears the argmax keys. */
int rngd_decode_embed(const rngd_model_t* m, const rngd_decode_io_t* io, rngd_stream_t stream);
/* Layers [layer0, layer1) of the batched decode step, updating the cache at
 * pos[b]; io->kcache/vcache hold exactly those layers (layer1 - layer0 <=
 * io->kv_layers), like the per-group cache of the reference (replaces DecodeModel.forward over one layer group,
 * kernels/decode_batch.py:73-109, called from engines/decode_batch.py:436-439). */
int rngd_decode_layers(const rngd_model_t* m, const rngd_decode_io_t* io, int layer0, int layer1,
                       rngd_stream_t stream);
/* io->x (fp32 [B][H]) already holds the residual stream, written by the caller: writes
 * layer0's first operand (x * n1[layer0], hi/lo) and its sums of squares and clears the
 * argmax keys, so rngd_decode_layers can start at layer0 from a given hidden state
 * (replaces the x input of DecodeModel.forward, kernels/decode_batch.py:100-109). */
int rngd_decode_begin(const rngd_model_t* m, const rngd_decode_io_t* io, int layer0, rngd_stream_t stream);
/* Final norm + lm_head + first-max argmax into io->next; logits kept in
 * io->logits (engines/decode_batch.py:440 and greedy_tokens 162-171).
 * The layer GEMMs and the lm_head run on tcgen05 tensor cores. */
int rngd_decode_lmhead(const rngd_model_t* m, const rngd_decode_io_t* io, rngd_stream_t stream);

/* toks[b] = next[b]; pos[b] += 1 for b < B: feeds a greedy step's output back as
 * the next step's input on the device, so multi-step decoding needs no host
 * round trip (the reference loops step() through the host,
 * src/rngd_pd/serving/cluster.py:1374-1380). */
int rngd_decode_advance(const rngd_decode_io_t* io, rngd_stream_t stream);

/* Final norm + lm_head + first-max argmax for `rows` (<= 16) rows of x (fp32,
 * row stride ldx), e.g. the last prompt position of a prefill
 * (engines/prefill_full.py:265-270 _next_token).  act: zeroed bf16 [32][H];
 * ss: fp32 [H/128][16]; logits [rows][V]; best [16]; next [rows]; partial /
 * counters from rngd_lmhead_workspace (both zeroed once, one pair per caller). */
int rngd_lmhead_rows(const rngd_model_t* m, const float* x, int ldx, int rows, void* act, float* ss, float* logits,
                     uint64_t* best, int32_t* next, float* partial, int32_t* counters, rngd_stream_t stream);
int rngd_lmhead_workspace(const rngd_model_t* m, size_t* partial_floats, size_t* counters);

/* ------------------------------------------------------------- prefill_full
 * One prompt of P tokens padded to a bucket of C tokens (C a multiple of 128,
 * engines/prefill_full.py:168-208 buckets), all 32 layers, K/V emitted in the
 * prefill layout kv [kv_layers][2][NKV][S][HD] (K then V per layer; positions
 * >= P are left as the caller zeroed them, engines/prefill_full.py:319-335).
 * Operand buffers hold 2C bf16 rows: hi of token t at row t, lo at row C + t. */
typedef struct rngd_prefill_io {
  int32_t C;            /* bucket width (tokens computed) */
  int32_t P;            /* prompt tokens (rows >= P are padding) */
  int32_t S;            /* KV width in positions (>= P) */
  int32_t kv_layers;    /* layers held by kv (the group's block) */
  void* kv;             /* bf16 [kv_layers][2][NKV][S][HD], first layer = layer0 of the call */
  const int32_t* toks;  /* device [C] token ids (the prompt, padded) */
  float* x;             /* fp32 [C][H] residual stream */
  float* q;             /* C*NH*HD*4 bytes: the rotated queries as bf16 hi/lo rows [2][C][NH*HD] */
  void* act;            /* bf16 [2C][max(H, NH*HD)] operand of x * norm weight */
  void* act_o;          /* bf16 [2C][NH*HD] attention-output operand */
  void* act2;           /* bf16 [2C][M] down-projection operand (also V^T scratch during attention) */
  float* ss;            /* fp32 [H/128][C] per-128-column sums of squares of x */
  float* partial;       /* fp32 split-K scratch, rngd_prefill_workspace() floats */
  int32_t* counters;    /* int32 tile counters, rngd_prefill_workspace() entries, zeroed once */
  int32_t operand_lo;   /* 1: GEMM operands as bf16 hi + lo rows (W*hi + W*lo, fp32-level accuracy);
                           0: the hi row alone, one bf16 operand as the reference's graph takes bf16
                           activations (kernels/prefill_full.py:56-76) at half the tensor work */
} rngd_prefill_io_t;

int rngd_prefill_workspace(const rngd_model_t* m, int C, size_t* partial_floats, size_t* counters);
/* x = embed[toks]; act = hi/lo(x * n1[0]); ss (prompt embedding, engines/prefill_full.py:356-357). */
int rngd_prefill_embed(const rngd_model_t* m, const rngd_prefill_io_t* io, rngd_stream_t stream);
/* io->x (fp32 [C][H]) already holds the residual stream, written by the caller: layer0's
 * first operand and sums of squares (replaces the x input of PrefillModel.forward,
 * kernels/prefill_full.py:79-94). */
int rngd_prefill_begin(const rngd_model_t* m, const rngd_prefill_io_t* io, int layer0, rngd_stream_t stream);
/* Layers [layer0, layer1) of the prefill (replaces PrefillModel.forward over one layer
 * group, kernels/prefill_full.py:56-94, called from engines/prefill_full.py:210-214). */
int rngd_prefill_layers(const rngd_model_t* m, const rngd_prefill_io_t* io, int layer0, int layer1,
                        rngd_stream_t stream);

/* ------------------------------------------------------ KV handoff (NVLink)
 * Replaces the host-staged KV transports of the connector
 * (connector/rngd_kv.py:122-166 save_kv_layer / wait_for_layer_load over
 * connector/transport.py:80-101 ShmTransport) with peer-to-peer stores.
 * Buffers shared across processes are cudaMalloc allocations exported with
 * CUDA IPC (the handshake hooks connector/transport.py:55-60 carry the handles). */
/* cudaMalloc `bytes` (zeroed) and its IPC handle (rngd_ipc_handle_size() bytes). */
int rngd_ipc_alloc(size_t bytes, void** ptr, void* handle);
int rngd_ipc_free(void* ptr);
/* Map a peer process's buffer (cudaIpcOpenMemHandle, lazy peer access). */
int rngd_ipc_open(const void* handle, void** ptr);
int rngd_ipc_close(void* ptr);
int rngd_ipc_handle_size(void);
/* Enable direct access from `device` to `peer` (one process driving both GPUs). */
int rngd_peer_enable(int device, int peer);
/* The copy engine moving `bytes` from src on src_device to dst on dst_device (cudaMemcpyPeerAsync,
 * direct over NVLink once rngd_peer_enable(src_device, dst_device) ran): the comparator the fused
 * handoff is measured against.  It has no counterpart in the reference, whose handoff is host-staged. */
int rngd_peer_copy(void* dst, int dst_device, const void* src, int src_device, size_t bytes, rngd_stream_t stream);
/* Pinned host memory mapped into the device address space (status words). */
int rngd_host_alloc_mapped(size_t bytes, void** host, void** dev);
int rngd_host_free(void* host);
/* Move positions [0, tokens) of layers [layer0, layer1) of one request's cache
 * into lane `lane` of dst_k / dst_v (decode layout [L][Bcap][NKV][S][HD] bf16,
 * local or peer memory), then publish flags[l] = seq (int64, system-scope
 * release) for each moved layer.  Source: src_k / src_v point at layer0's K and
 * V blocks ([NKV][S][HD] bf16 each, local) and successive layers are
 * src_layer_stride elements apart (2*NKV*S*HD for the prefill layout
 * [L][2][NKV][S][HD]).  done: a zeroed uint32 on the sending device, one per
 * stream of handoffs. */
int rngd_kv_handoff(const void* src_k, const void* src_v, size_t src_layer_stride, void* dst_k, void* dst_v, int L,
                    int NKV, int S, int HD, int tokens, int lane, int Bcap, int layer0, int layer1, uint32_t* done,
                    int64_t* flags, int64_t seq, rngd_stream_t stream);
/* One request of a batched handoff: its layer0 K / V blocks (as in rngd_kv_handoff),
 * the decode lane it lands in, how many leading positions move, and the lease's
 * sequence number published in the lane's flags. */
#define RNGD_KV_MAX_BATCH 16
typedef struct {
  const void* src_k;
  const void* src_v;
  int lane;
  int tokens;
  int64_t seq;
} rngd_kv_item_t;
/* rngd_kv_handoff for 1..RNGD_KV_MAX_BATCH requests (distinct lanes) into one
 * receiver in a single launch.  flags: the receiver's whole [Bcap][L] int64 flag
 * array; done: n zeroed uint32 counters on the sending device (one set per stream). */
int rngd_kv_handoff_batch(const rngd_kv_item_t* items, int n, size_t src_layer_stride, void* dst_k, void* dst_v,
                          int L, int NKV, int S, int HD, int Bcap, int layer0, int layer1, uint32_t* done,
                          int64_t* flags, rngd_stream_t stream);
/* Copies n int64 handoff flags (device memory) into `host` (pinned) on `stream` and waits for the
 * copy: the receiver's host poll of which layers have landed, one call per poll for every lane
 * (the reference's receiver polls its store the same way, connector/transport.py:80-101). */
int rngd_kv_read_flags(const int64_t* flags, int64_t* host, size_t n, rngd_stream_t stream);
/* Bounded device wait until flags[l] >= seq for l in [layer0, layer1): writes 0,
 * or RNGD_ERR_TIMEOUT's wait code 4 after timeout_ns (<= 10 s), to *status
 * (e.g. host-mapped); later work on `stream` is ordered after the arrival. */
int rngd_kv_wait(const int64_t* flags, int layer0, int layer1, int64_t seq, int64_t timeout_ns, int32_t* status,
                 rngd_stream_t stream);

/* ------------------------------------------------------ kernel-level ops
 * Exposed for the parity tests and for hosts that build their own step. */
/* Y[b][n] (+)= sum_k W[n][k] * X[b][k]; W bf16 [N][K] row-major, X/Y fp32,
 * b < B <= 16, K % 8 == 0 (CUDA-core path, fp32 accumulation). */
int rngd_gemv_bf16(const void* W, int N, int K, const float* X, int ldx, int B, float* Y, int ldy,
                   int accumulate, rngd_stream_t stream);
/* Tensor-core form of the same op (the one the decode step uses): Y[b][n] +=
 * sum_k W[n][k] * X[b][k] through tcgen05 with the fp32 X split into bf16
 * hi + lo operand rows.  act: zeroed bf16 scratch [32][K]; partial/counters:
 * split-K scratch of rngd_tc_gemv_workspace() (both zeroed once; one pair
 * per (N, K) shape).
 * prep = 0 reuses the operand already in act (X is not read).
 * N % 128 == 0, K % 64 == 0, B <= 16. */
int rngd_tc_gemv(const void* W, int N, int K, const float* X, int ldx, int B, float* Y, int ldy, void* act,
                 float* partial, int32_t* counters, int prep, rngd_stream_t stream);
int rngd_tc_gemv_workspace(int N, int K, size_t* partial_floats, size_t* counters);
/* Diagnostics, compiled in only by `make TRACE=1` (otherwise a non-NULL trace returns
 * RNGD_ERR_UNSUPPORTED): when trace != NULL, later rngd_tc_gemv launches record per CTA sixteen
 * %globaltimer slots (ns) [start, operand ready, last weight TMA issued, last stage
 * arrived, last MMA committed, last accumulator ready, epilogue done, end, then five
 * steps of the last segment's epilogue] into trace[cta*16 ..] (device memory,
 * >= 16 * SM count entries).  rngd_tc_gemm_tokens launches record into the same buffer their
 * own slots [start, TMA past the dependency wait, first full stage, last MMA committed, last
 * unit's accumulator ready / pieces acquired / epilogue done, first accumulator ready, last
 * unit's owner count, this CTA's slot in it, epilogue past the dependency wait]. */
int rngd_tc_gemv_trace(uint64_t* trace);
/* Diagnostics (TRACE=1 builds only, as above): the next `launches` decode or prefill GEMM
 * launches record their sixteen slots per CTA into consecutive blocks trace[i*1024*16 ..] (device
 * memory, launches * 16384 entries); NULL turns it off. */
int rngd_trace_decode_gemms(uint64_t* trace, int launches);
/* Token-tile form (the prefill GEMM): Y[t][n] += sum_k W[n][k] * X[t][k] for
 * C tokens (C % 128 == 0) on tcgen05, X fp32 [C][K] split into bf16 hi/lo rows
 * of act (zeroed bf16 scratch [2C][K]); partial/counters from
 * rngd_tc_gemm_tokens_workspace(); prep = 0 reuses the operand already in act. */
int rngd_tc_gemm_tokens(const void* W, int N, int K, const float* X, int C, float* Y, void* act, float* partial,
                        int32_t* counters, int prep, rngd_stream_t stream);
int rngd_tc_gemm_tokens_workspace(int N, int K, int C, size_t* partial_floats, size_t* counters);
/* out[r][k] = x[r][k] / sqrt(mean_k x^2 + eps) * w[k] (kernels/decode_batch.py:130). */
int rngd_rmsnorm_f32(const float* x, int R, int H, const float* w, float eps, float* out,
                     rngd_stream_t stream);
/* Split-S decode attention for one layer: q fp32 [B][NH*HD] (already rotated),
 * caches bf16 [Bcap][NKV][S][HD] of that layer, positions [B] -> ao fp32
 * [B][NH*HD] (kernels/decode_batch.py:83-85 with the mask of :153). */
int rngd_attn_decode(const float* q, const void* kc, const void* vc, const int32_t* pos, int B,
                     int Bcap, int NH, int NKV, int HD, int S, float* part, float* ao,
                     rngd_stream_t stream);

/* Allocation-free form of rngd_attn_decode, for callers that cannot call
 * cudaMalloc: code running inside someone else's CUDA-graph capture or memory
 * pool, or a host whose allocator owns all device memory.  It has no
 * counterpart in the reference.  The chunk partials live in a scratch array
 * built into this library (2,129,920 bytes on every GPU that loads it, held
 * until exit): B * NH * S/128 must be <= 4096 (B=16, NH=32 allows S <= 1024),
 * larger requests return RNGD_ERR_ARG.  The caller still passes q, the caches,
 * positions and the output ao.  Nothing in the scratch needs to start at zero
 * (every record is written before it is read), but every call shares it:
 * calls that may overlap on the GPU (other streams, other threads) race, so
 * order them on one stream.  The first call on a device looks up the scratch
 * address with cudaGetSymbolAddress (which may load the module); make that
 * first call before any stream capture.  No cudaMalloc/cudaFree is made. */
int rngd_attn_decode_noalloc(const float* q, const void* kc, const void* vc, const int32_t* pos, int B,
                             int Bcap, int NH, int NKV, int HD, int S, float* ao, rngd_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* RNGD_B200_H */
