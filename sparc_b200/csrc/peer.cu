// Parameter-gradient all-reduce over NVLink peer memory for batch-sharded data parallelism
// (the one exchange step of the SPARC layers, whose gradients are a few thousand floats per
// layer: a latency-bound collective).
//
// Every rank holds one buffer, mapped into every other rank's address space by CUDA IPC:
//   epoch [ctas] u32              this rank's launch count, one word per CTA
//   inbox [2][world][cap] u64     inbox[e & 1][src]: src's gradients of epoch e, each float in
//                                 the low half of an 8-byte word whose high half holds e
// One launch, grid = ceil(total / 1024) CTAs of 256 threads, CTA c owning the flat gradient
// elements [1024 c, 1024 c + 1024): it gathers its slice from the gradient tensors (up to 64
// segments) and stores each value with the epoch e as one 8-byte word into inbox[e & 1][rank] of
// EVERY rank's buffer (peer stores over NVLink; a naturally aligned 8-byte store is single-copy
// atomic, so a reader that sees e in a word sees the value stored with it: no fence, no flag).
// Then every thread polls, in its own inbox, its elements' words from every rank until they carry
// e (bounded: a wait that runs out sets a status bit and the sum proceeds), and sums them in rank
// order into the gradient tensors: every rank computes the identical sum (deterministic,
// rank-independent). Epoch parity double-buffers the inbox: a peer can be one launch ahead (it
// has seen this rank's push of epoch e) but not two (epoch e+2 needs this rank's push of e+1,
// which starts only after this launch, including its reads of inbox[e & 1], has finished on this
// stream). Each CTA keeps its own epoch word, so no CTA of a launch can see another's update.
#include "common.cuh"
#include "sparc_b200.h"
#include "timing.cuh"

#include <cstdio>
#include <cstring>

namespace sparc {

constexpr int kPeerThreads = 256;
constexpr int kPeerPerThread = 4;
constexpr int kPeerSlice = kPeerThreads * kPeerPerThread;
constexpr int kPeerMax = SPARC_PEER_MAX_RANKS;
constexpr int kPeerMaxSeg = SPARC_PEER_MAX_SEGMENTS;
constexpr unsigned kStatusPeerTimeout = 8u;

struct PeerLayout {
  long long ctas, cap;
  size_t epoch, inbox, total;
};

static PeerLayout peer_layout(int world, long long total) {
  PeerLayout L;
  L.ctas = (total + kPeerSlice - 1) / kPeerSlice;
  L.cap = L.ctas * kPeerSlice;
  L.epoch = 0;
  L.inbox = ((size_t)L.ctas * 4 + 255) & ~size_t(255);
  L.total = L.inbox + 2 * (size_t)world * (size_t)L.cap * 8;
  return L;
}

struct PeerParams {
  float* seg[kPeerMaxSeg];
  long long off[kPeerMaxSeg + 1];  // prefix offsets of the segments in the flat vector
  int nseg;
  long long total;
  unsigned char* base[kPeerMax];   // every rank's buffer, as mapped here (own included)
  long long ctas, cap;
  unsigned long long epoch_off, inbox_off;
  int world, rank;
  float scale;
  unsigned max_spin;
  unsigned* status;
  int skip_publish;                // failure test: push nothing (peers' waits run out)
};

__global__ void __launch_bounds__(kPeerThreads) peer_allreduce_kernel(const __grid_constant__ PeerParams p) {
  pdl_wait();  // the gradients come from the previous kernels
  const int c = blockIdx.x, tid = threadIdx.x;
  __shared__ unsigned s_epoch;
  __shared__ long long s_off[kPeerMaxSeg + 1];
  unsigned* my_epoch = reinterpret_cast<unsigned*>(p.base[p.rank] + p.epoch_off) + c;
  if (tid == 0) s_epoch = *my_epoch + 1u;
  for (int i = tid; i <= p.nseg; i += kPeerThreads) s_off[i] = p.off[i];
  __syncthreads();
  const unsigned e = s_epoch;
  const int par = (int)(e & 1u);
  const long long first = (long long)c * kPeerSlice;

  // gather this CTA's slice (segment of each element by a scan over the prefix offsets)
  float v[kPeerPerThread];
  int segi[kPeerPerThread];
  long long loc[kPeerPerThread];
#pragma unroll
  for (int u = 0; u < kPeerPerThread; ++u) {
    const long long i = first + u * kPeerThreads + tid;
    v[u] = 0.0f;
    segi[u] = -1;
    if (i < p.total) {
      int s = 0;
      while (s + 1 < p.nseg && s_off[s + 1] <= i) ++s;
      segi[u] = s;
      loc[u] = i - s_off[s];
      v[u] = p.seg[s][loc[u]];
    }
  }
  // push each value with the epoch into inbox[par][rank] of every rank
  const unsigned long long tag = (unsigned long long)e << 32;
  if (!p.skip_publish) {
    for (int r = 0; r < p.world; ++r) {
      unsigned long long* dst = reinterpret_cast<unsigned long long*>(p.base[r] + p.inbox_off) +
                                ((long long)par * p.world + p.rank) * p.cap + first;
#pragma unroll
      for (int u = 0; u < kPeerPerThread; ++u)
        if (segi[u] >= 0) st_relaxed_sys_u64(dst + u * kPeerThreads + tid, tag | __float_as_uint(v[u]));
    }
  }
  // wait for every rank's words of epoch e and sum them in rank order (identical on every rank)
  const unsigned long long* in =
      reinterpret_cast<const unsigned long long*>(p.base[p.rank] + p.inbox_off) + (long long)par * p.world * p.cap + first;
  bool late = false;
#pragma unroll
  for (int u = 0; u < kPeerPerThread; ++u) {
    if (segi[u] < 0) continue;
    float s = 0.0f;
    for (int r = 0; r < p.world; ++r) {
      const unsigned long long* w = in + (long long)r * p.cap + u * kPeerThreads + tid;
      unsigned long long got = ld_relaxed_sys_u64(w);
      unsigned it = 0;
      while (!late && (unsigned)(got >> 32) != e) {
        if (++it >= p.max_spin) {
          late = true;  // (later words of this thread do not wait again)
          break;
        }
        __nanosleep(32);
        got = ld_relaxed_sys_u64(w);
      }
      s += __uint_as_float((unsigned)got);
    }
    p.seg[segi[u]][loc[u]] = s * p.scale;
  }
  if (late) atomicOr(p.status, kStatusPeerTimeout);
  __syncthreads();  // every thread of the CTA is done with this epoch's words
  if (tid == 0) *my_epoch = e;
}

static thread_local char g_peer_err[256];

static int peer_fail(int code, const char* msg) {
  snprintf(g_peer_err, sizeof(g_peer_err), "%s", msg);
  return code;
}

static int peer_cuda(cudaError_t e) {
  if (e == cudaSuccess) return SPARC_OK;
  cudaGetLastError();
  return peer_fail(SPARC_ERR_LAUNCH, cudaGetErrorString(e));
}

}  // namespace sparc

using namespace sparc;

extern "C" {

const char* sparc_peer_last_error(void) { return g_peer_err; }

size_t sparc_peer_buffer_bytes(int world, long long total) {
  if (world < 1 || world > kPeerMax || total <= 0) return 0;
  return peer_layout(world, total).total;
}

int sparc_peer_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (ptr == nullptr || ipc_handle == nullptr || bytes == 0) return peer_fail(SPARC_ERR_ARG, "null pointer or size");
  void* p = nullptr;
  int rc = peer_cuda(cudaMalloc(&p, bytes));
  if (rc != SPARC_OK) return rc;
  rc = peer_cuda(cudaMemset(p, 0, bytes));
  cudaIpcMemHandle_t h;
  if (rc == SPARC_OK) rc = peer_cuda(cudaIpcGetMemHandle(&h, p));
  if (rc != SPARC_OK) {
    cudaFree(p);
    return rc;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return SPARC_OK;
}

int sparc_peer_buffer_open(const void* ipc_handle, void** ptr) {
  if (ptr == nullptr || ipc_handle == nullptr) return peer_fail(SPARC_ERR_ARG, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return peer_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int sparc_peer_buffer_close(void* ptr) { return peer_cuda(cudaIpcCloseMemHandle(ptr)); }

int sparc_peer_buffer_free(void* ptr) { return peer_cuda(cudaFree(ptr)); }

int sparc_peer_allreduce(const SparcPeerAllreduceArgs* a, void* stream) {
  NvtxRange nvtx(__func__);
  if (a == nullptr) return peer_fail(SPARC_ERR_ARG, "null args");
  if (a->world < 1 || a->world > kPeerMax || a->rank < 0 || a->rank >= a->world)
    return peer_fail(SPARC_ERR_ARG, "world must be 1..8 and rank in [0, world)");
  if (a->nseg < 1 || a->nseg > kPeerMaxSeg) return peer_fail(SPARC_ERR_ARG, "1..64 segments");
  if (a->status == nullptr) return peer_fail(SPARC_ERR_ARG, "null status");
  PeerParams p;
  long long total = 0;
  p.off[0] = 0;
  for (int s = 0; s < a->nseg; ++s) {
    if (a->segments[s] == nullptr || a->counts[s] <= 0) return peer_fail(SPARC_ERR_ARG, "empty or null segment");
    p.seg[s] = a->segments[s];
    total += a->counts[s];
    p.off[s + 1] = total;
  }
  if (total != a->total) return peer_fail(SPARC_ERR_ARG, "segment counts do not add up to the buffer's total");
  for (int r = 0; r < a->world; ++r) {
    if (a->buffers[r] == nullptr) return peer_fail(SPARC_ERR_ARG, "null peer buffer");
    p.base[r] = static_cast<unsigned char*>(a->buffers[r]);
  }
  const PeerLayout L = peer_layout(a->world, total);
  p.nseg = a->nseg;
  p.total = total;
  p.ctas = L.ctas;
  p.cap = L.cap;
  p.epoch_off = L.epoch;
  p.inbox_off = L.inbox;
  p.world = a->world;
  p.rank = a->rank;
  p.scale = a->scale;
  p.max_spin = a->max_spin ? a->max_spin : (1u << 24);
  p.status = a->status;
  p.skip_publish = a->inject_skip_publish;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)L.ctas, 1, 1);
  cfg.blockDim = dim3(kPeerThreads, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {&p};
  TimedLaunch tl(kTimePeerAllreduce, s);
  return peer_cuda(cudaLaunchKernelExC(&cfg, (const void*)peer_allreduce_kernel, args));
}

}  // extern "C"
