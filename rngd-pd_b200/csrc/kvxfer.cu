// KV handoff prefill GPU -> decode GPU over NVLink (peer-to-peer stores).
//
// Replaces the reference's host-staged handoff: download, bf16 wire encoding,
// /dev/shm file, decode, upload (src/rngd_pd/connector/rngd_kv.py:122-166,
// src/rngd_pd/connector/transport.py:29-101, src/rngd_pd/serving/cluster.py:438-467).
// A request's cache travels in the prefill layout [L][2][NKV][S][HD] (K then V per
// layer); the decode cache keeps K and V as [L][Bcap][NKV][S][HD].  Moving
// layers [l0, l1) of one request's first `tokens` positions into decode lane `lane`
// is therefore a set of contiguous tokens*HD-element runs, one per (layer, K|V, head):
// one fused kernel (a CTA per 32 KB chunk of a run, up to 16 requests per launch)
// reads them from local HBM
// (16-byte loads) and stores them straight into the destination, which may be a
// peer GPU's memory mapped by CUDA IPC or peer access, so pack, transfer and unpack
// are one pass.
//
// Completion fence: every CTA fences after its stores and counts itself into its
// request's counter; the CTA that completes a request's count issues one fence.sc.sys
// and then publishes flags[l] = seq for each moved layer with relaxed system-scope
// stores (a fence followed by strong writes is a release of each of them; the
// "threadfence reduction" pattern), so a reader that observes a flag with acquire
// semantics sees all the request's bytes.  One fence, not a release store per layer:
// every system-scope release waits for the previous one, and 32 of them in a row cost
// ~50 us per launch.  The reader's wait is a bounded device loop that reports a
// status; it never traps or spins forever.
#include "tc.cuh"

namespace rngd {

constexpr int kXferThreads = 256;
constexpr int kXferVec = 8;                                    // 16-byte vectors per thread per chunk
constexpr unsigned kXferChunk = kXferThreads * kXferVec;       // 2048 vectors = 32 KB

// A batch of requests moved by one launch into lanes of one receiver's cache.
struct XferBatch {
  const uint4* src_k[RNGD_KV_MAX_BATCH];
  const uint4* src_v[RNGD_KV_MAX_BATCH];
  long long seq[RNGD_KV_MAX_BATCH];
  unsigned run_vec[RNGD_KV_MAX_BATCH];   // 16-byte vectors of one run (tokens * HD * 2 / 16)
  unsigned cpr[RNGD_KV_MAX_BATCH];       // chunks per run
  unsigned first[RNGD_KV_MAX_BATCH + 1]; // first CTA of each request; first[n] = grid
  int lane[RNGD_KV_MAX_BATCH];
  int n;
};

// One CTA per chunk: 32 KB of one run of one request.  A run is (layer, K|V, head): the
// first `tokens` positions of one head, run_vec contiguous 16-byte vectors in both layouts
// (heads sit head_vec vectors apart).  The CTA -> (request, run, part) split costs a scan
// over at most 16 entries and two divisions per CTA; the per-vector work is an add, a load
// and a store, with kXferVec independent loads in flight per thread.
//
// Completion: each CTA fences at gpu scope (the counters live on this GPU) and counts itself
// into its request's counter; the CTA that completes a request fences once at system scope
// and then writes that request's layer flags with relaxed system-scope stores, so a reader
// acquiring a flag sees every byte of the request.
__global__ void __launch_bounds__(kXferThreads) kv_handoff_kernel(const __grid_constant__ XferBatch b,
                                                                  long src_stride_vec, uint4* __restrict__ dst_k,
                                                                  uint4* __restrict__ dst_v, unsigned head_vec,
                                                                  int NKV, int L, int Bcap, int layer0, int layer1,
                                                                  unsigned int* __restrict__ done,
                                                                  long long* __restrict__ flags) {
  grid_dep_wait();
  int r = 0;
  while (r + 1 < b.n && blockIdx.x >= b.first[r + 1]) r++;
  const unsigned cta = blockIdx.x - b.first[r];
  const unsigned run = cta / b.cpr[r], part = cta - run * b.cpr[r];
  const unsigned h = run % (unsigned)NKV, lkv = run / (unsigned)NKV, lr = lkv >> 1;
  const bool isv = lkv & 1u;
  const unsigned run_vec = b.run_vec[r];
  const uint4* s = (isv ? b.src_v[r] : b.src_k[r]) + (long)lr * src_stride_vec + (long)h * head_vec;
  uint4* d = (isv ? dst_v : dst_k) + (((long)(layer0 + (int)lr) * Bcap + b.lane[r]) * NKV + h) * (long)head_vec;
  const unsigned o0 = part * kXferChunk + threadIdx.x;
  uint4 v[kXferVec];
#pragma unroll
  for (int j = 0; j < kXferVec; j++) {
    const unsigned o = o0 + j * kXferThreads;
    if (o < run_vec) v[j] = ldg_nc_v4(s + o);
  }
#pragma unroll
  for (int j = 0; j < kXferVec; j++) {
    const unsigned o = o0 + j * kXferThreads;
    if (o < run_vec) d[o] = v[j];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(done + r, 1u);
    if (prev == b.first[r + 1] - b.first[r] - 1) {
      __threadfence_system();
      long long* f = flags + (long)b.lane[r] * L;
      for (int l = layer0; l < layer1; l++)
        asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(f + l), "l"(b.seq[r]) : "memory");
      done[r] = 0u;  // ready for the next handoff on this stream
    }
  }
}

// Bounded wait for flags[l] >= seq for l in [layer0, layer1): status 0 when all
// arrived, ST_FLAG_WAIT after timeout_ns.  The status goes to a word the host
// can read without synchronising (host-mapped) and is also returned in *dev_status.
__global__ void kv_wait_kernel(const long long* __restrict__ flags, int layer0, int layer1, long long seq,
                               long long timeout_ns, int* status) {
  if (threadIdx.x != 0) return;
  const uint64_t t0 = globaltimer();
  int st = 0;
  for (int l = layer0; l < layer1 && st == 0; l++) {
    for (;;) {
      long long v;
      asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(flags + l) : "memory");
      if (v >= seq) break;
      if ((long long)(globaltimer() - t0) > timeout_ns) {
        st = ST_FLAG_WAIT;
        break;
      }
      __nanosleep(256);
    }
  }
  asm volatile("st.volatile.global.b32 [%0], %1;" ::"l"(status), "r"(st) : "memory");
  __threadfence_system();
}

}  // namespace rngd

using namespace rngd;

extern "C" int rngd_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  RNGD_REQUIRE(ptr && handle && bytes > 0, "ipc_alloc: bad arguments");
  void* p = nullptr;
  RNGD_TRY(check_cuda(cudaMalloc(&p, bytes), "cudaMalloc (IPC-exportable buffer)"));
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle((cudaIpcMemHandle_t*)handle, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return check_cuda(e, "cudaIpcGetMemHandle");
  }
  *ptr = p;
  return RNGD_OK;
}

extern "C" int rngd_ipc_free(void* ptr) { return check_cuda(cudaFree(ptr), "cudaFree (IPC buffer)"); }

extern "C" int rngd_ipc_open(const void* handle, void** ptr) {
  RNGD_REQUIRE(handle && ptr, "ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return check_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

extern "C" int rngd_ipc_close(void* ptr) { return check_cuda(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle"); }

extern "C" int rngd_ipc_handle_size(void) { return (int)sizeof(cudaIpcMemHandle_t); }

extern "C" int rngd_peer_enable(int device, int peer) {
  int can = 0;
  RNGD_TRY(check_cuda(cudaDeviceCanAccessPeer(&can, device, peer), "cudaDeviceCanAccessPeer"));
  RNGD_REQUIRE(can, "device %d cannot access device %d directly", device, peer);
  int cur = 0;
  RNGD_TRY(check_cuda(cudaGetDevice(&cur), "cudaGetDevice"));
  RNGD_TRY(check_cuda(cudaSetDevice(device), "cudaSetDevice"));
  cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    e = cudaSuccess;
  }
  cudaSetDevice(cur);
  return check_cuda(e, "cudaDeviceEnablePeerAccess");
}

extern "C" int rngd_host_alloc_mapped(size_t bytes, void** host, void** dev) {
  RNGD_REQUIRE(host && dev && bytes > 0, "host_alloc_mapped: bad arguments");
  RNGD_TRY(check_cuda(cudaHostAlloc(host, bytes, cudaHostAllocMapped | cudaHostAllocPortable), "cudaHostAlloc"));
  memset(*host, 0, bytes);
  return check_cuda(cudaHostGetDevicePointer(dev, *host, 0), "cudaHostGetDevicePointer");
}

extern "C" int rngd_host_free(void* host) { return check_cuda(cudaFreeHost(host), "cudaFreeHost"); }

extern "C" int rngd_kv_handoff_batch(const rngd_kv_item_t* items, int n, size_t src_layer_stride, void* dst_k,
                                     void* dst_v, int L, int NKV, int S, int HD, int Bcap, int layer0, int layer1,
                                     uint32_t* done, int64_t* flags, rngd_stream_t stream) {
  RNGD_REQUIRE(items && 1 <= n && n <= RNGD_KV_MAX_BATCH, "kv_handoff: 1..%d requests per launch, got %d",
               RNGD_KV_MAX_BATCH, n);
  RNGD_REQUIRE(dst_k && dst_v && done && flags, "kv_handoff: null pointer");
  RNGD_REQUIRE(0 <= layer0 && layer0 < layer1 && layer1 <= L, "kv_handoff: layers [%d, %d) outside [0, %d)",
               layer0, layer1, L);
  RNGD_REQUIRE(NKV > 0 && HD > 0 && S > 0 && (HD * 2) % 16 == 0 && src_layer_stride % 8 == 0 &&
                   ((uintptr_t)dst_k | (uintptr_t)dst_v) % 16 == 0,
               "kv_handoff: HD*2 and the layer stride must be 16-byte multiples, buffers 16-byte aligned");
  const long head_vec = (long)S * HD * 2 / 16;
  RNGD_REQUIRE(head_vec < (1l << 31), "kv_handoff: S*HD too large");
  XferBatch b;
  memset(&b, 0, sizeof(b));
  b.n = n;
  long grid = 0;
  for (int i = 0; i < n; i++) {
    const rngd_kv_item_t& it = items[i];
    RNGD_REQUIRE(it.src_k && it.src_v && ((uintptr_t)it.src_k | (uintptr_t)it.src_v) % 16 == 0,
                 "kv_handoff: request %d: null or unaligned source", i);
    RNGD_REQUIRE(0 <= it.lane && it.lane < Bcap, "kv_handoff: request %d: lane %d outside 0..%d", i, it.lane,
                 Bcap - 1);
    RNGD_REQUIRE(0 < it.tokens && it.tokens <= S, "kv_handoff: request %d: tokens %d outside 1..S=%d", i, it.tokens,
                 S);
    for (int j = 0; j < i; j++)
      RNGD_REQUIRE(items[j].lane != it.lane, "kv_handoff: requests %d and %d share lane %d", j, i, it.lane);
    const long run_vec = (long)it.tokens * HD * 2 / 16;
    const long cpr = (run_vec + kXferChunk - 1) / kXferChunk;
    b.src_k[i] = (const uint4*)it.src_k;
    b.src_v[i] = (const uint4*)it.src_v;
    b.seq[i] = (long long)it.seq;
    b.run_vec[i] = (unsigned)run_vec;
    b.cpr[i] = (unsigned)cpr;
    b.lane[i] = it.lane;
    b.first[i] = (unsigned)grid;
    grid += cpr * 2 * NKV * (layer1 - layer0);
    RNGD_REQUIRE(grid < (1l << 31), "kv_handoff: batch too large for one launch");
  }
  b.first[n] = (unsigned)grid;
  return launch_pdl(kv_handoff_kernel, dim3((unsigned)grid), dim3(kXferThreads), 0, (cudaStream_t)stream,
                    "kv_handoff_kernel", b, (long)(src_layer_stride / 8), (uint4*)dst_k, (uint4*)dst_v,
                    (unsigned)head_vec, NKV, L, Bcap, layer0, layer1, (unsigned int*)done, (long long*)flags);
}

extern "C" int rngd_kv_handoff(const void* src_k, const void* src_v, size_t src_layer_stride, void* dst_k,
                               void* dst_v, int L, int NKV, int S, int HD, int tokens, int lane, int Bcap, int layer0,
                               int layer1, uint32_t* done, int64_t* flags, int64_t seq, rngd_stream_t stream) {
  RNGD_REQUIRE(flags, "kv_handoff: null flags");
  rngd_kv_item_t it;
  it.src_k = src_k;
  it.src_v = src_v;
  it.lane = lane;
  it.tokens = tokens;
  it.seq = seq;
  // the single-request form takes the lane's own flag row
  return rngd_kv_handoff_batch(&it, 1, src_layer_stride, dst_k, dst_v, L, NKV, S, HD, Bcap, layer0, layer1, done,
                               flags - (long)lane * L, stream);
}

extern "C" int rngd_peer_copy(void* dst, int dst_device, const void* src, int src_device, size_t bytes,
                              rngd_stream_t stream) {
  RNGD_REQUIRE(dst != nullptr && src != nullptr, "peer_copy: null pointer");
  return check_cuda(cudaMemcpyPeerAsync(dst, dst_device, src, src_device, bytes, (cudaStream_t)stream),
                    "cudaMemcpyPeerAsync");
}

extern "C" int rngd_kv_read_flags(const int64_t* flags, int64_t* host, size_t n, rngd_stream_t stream) {
  RNGD_REQUIRE(flags != nullptr && host != nullptr && n > 0, "kv_read_flags: null or empty buffer");
  cudaStream_t s = (cudaStream_t)stream;
  RNGD_TRY(check_cuda(cudaMemcpyAsync(host, flags, n * sizeof(int64_t), cudaMemcpyDeviceToHost, s),
                      "cudaMemcpyAsync (handoff flags)"));
  return check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize (handoff flags)");
}

extern "C" int rngd_kv_wait(const int64_t* flags, int layer0, int layer1, int64_t seq, int64_t timeout_ns,
                            int32_t* status, rngd_stream_t stream) {
  RNGD_REQUIRE(flags && status, "kv_wait: null pointer");
  RNGD_REQUIRE(0 <= layer0 && layer0 < layer1, "kv_wait: bad layer range");
  RNGD_REQUIRE(timeout_ns > 0 && timeout_ns <= 10000000000ll, "kv_wait: timeout must be in (0, 10 s]");
  kv_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>((const long long*)flags, layer0, layer1, (long long)seq,
                                                     (long long)timeout_ns, (int*)status);
  return check_launch("kv_wait_kernel");
}
