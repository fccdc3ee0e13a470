// Real diagonal scan h_t = a_t h_{t-1} + b_t for B200 (sm_100a), forward and backward.
//
// Parity targets (Botwwt/sparc): _real_forward / _real_chunk_* forward/scan.py:622-698,
// _real_backward / _real_reverse_chunk_* backward/scan.py:35-128 (grad_a = lambda_t h_{t-1},
// grad_b = lambda_t). As in the reference, a is read in its own dtype and widened to float32
// (forward/scan.py:631), out and grad_b have b's dtype and grad_a has a's
// (backward/scan.py:815, 880); the recurrence and its carries are float32.
//
// Tile = (batch row b, chunk of kRealChunk = 32 tokens, K channels). Persistent CTAs, several per SM:
// a producer warp takes tiles from a global ticket counter (chunk-major order: forward from the
// first chunk, backward from the last; tickets claimed two at a time, the next pair requested a
// pair ahead so the atomic's latency stays off the copy path) and stages each tile of a, b (and
// grad_out) into a ring of S shared-memory stages with 2-D TMA tensor copies
// (cp.async.bulk.tensor, one box of up to 256 channels x 32 rows per instruction, completing on
// the stage's mbarrier; channels past D and rows past the last token arrive as zeros). A stage
// holds each array as [K / 256 boxes][32 rows][256 channels]. NT consumer threads own 2
// channels each. The
// consumers compose the tile's affine map (P, Q) from shared memory, obtain the carry-in by
// decoupled lookback, and replay the chunk from shared memory, storing straight from registers
// (each warp stores 128 or 256 contiguous bytes per row).
//
// Lookback without barriers: every channel of every tile has a status word of 64 bits,
// (float32 value, 32-bit tag = epoch << 2 | state), written with one relaxed 64-bit store. A
// reader that sees the tag of the current launch knows the value beside it is that launch's, so
// no fence or flag is needed, and each thread looks back for its own channels independently.
// State "inclusive": the value is the state (forward) / adjoint (backward) leaving the tile.
// State "aggregate": the value is P, and a second word (Q, same tag) holds Q. A tile publishes an
// aggregate only when its predecessor's inclusive is not yet visible when it looks. Every wait is
// bounded: a wait that runs out sets the launch status bit and continues with a zero carry.
//
// The backward replays h from the forward's saved carries (the state entering each chunk), so
// it reads a, b, grad_out once and never needs the forward output.
//
// Shapes whose rows are not whole 16-byte units (channels * element size), or pointers not
// 16-byte aligned, are staged by the producer warp with plain loads and shared-memory stores
// instead of tensor copies (same stage layout); everything else is the same kernel.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "sparc_b200.h"
#include "timing.cuh"

namespace sparc {

constexpr int kRealChunk = 32;  // tokens per tile (= the saved carry's granularity)
constexpr unsigned kTagAggregate = 1u;
constexpr unsigned kTagInclusive = 2u;

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long make_word(float v, unsigned tag) {
  return ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
}
__device__ __forceinline__ void mbar_arrive(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Two channels of a row in shared memory (or global memory) as floats, and back.
template <typename T>
struct Pair;
template <>
struct Pair<float> {
  static __device__ __forceinline__ float2 ld(const float* p) { return *reinterpret_cast<const float2*>(p); }
  static __device__ __forceinline__ void st(float* p, float2 v) { *reinterpret_cast<float2*>(p) = v; }
  static __device__ __forceinline__ void st1(float* p, float v) { *p = v; }
};
template <>
struct Pair<__nv_bfloat16> {
  static __device__ __forceinline__ float2 ld(const __nv_bfloat16* p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
  }
  static __device__ __forceinline__ void st(__nv_bfloat16* p, float2 v) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v.x, v.y);
  }
  static __device__ __forceinline__ void st1(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
};

struct RealParams {
  // [rows = B*T, D] 2-D maps, box {min(K, 256), 32} (tensor path): loads of a, b, grad_out and
  // stores of out (forward) / grad_a, grad_b (backward)
  CUtensorMap map_a, map_b, map_g, map_o, map_o2;
  const void* a;
  const void* b;
  const void* g;         // backward only
  void* out;             // forward: out; backward: grad_a
  void* out2;            // backward: grad_b
  float* last;           // forward, optional
  float* carry;          // [B, chunks, D]: forward writes, backward reads
  LaunchState* ls;
  unsigned long long* w1;  // [tiles, K] status words (inclusive value or aggregate P)
  unsigned long long* w2;  // [tiles, K] aggregate Q
  long long B, T, D;
  int chunks, nDB;
  long long tiles, per_chunk;  // tiles per chunk = B * nDB
  unsigned max_spin;
  int bulk;                    // tiles staged by TMA tensor copies (else plain loads)
  long long inject_unpublished;  // test hook: this forward tile never publishes (-1: none)
};

template <typename TA, typename TB, int NT, int S, bool BWD>
struct Cfg {
  static constexpr int C = kRealChunk;
  static constexpr int K = NT * 2;  // channels per tile
  static constexpr int BOXW = K < 256 ? K : 256;  // channels per TMA box
  static constexpr int NBOX = K / BOXW;
  static constexpr int ROW_A = K * (int)sizeof(TA);
  static constexpr int ROW_B = K * (int)sizeof(TB);
  static constexpr int ROW_G = BWD ? K * (int)sizeof(TB) : 0;
  static constexpr int OFF_B = C * ROW_A;
  static constexpr int OFF_G = OFF_B + C * ROW_B;
  static constexpr int OFF_H = OFF_G + C * ROW_G;         // backward: the carry entering the tile
  static constexpr int STAGE = OFF_H + (BWD ? K * 4 : 0);
  // element offset of (row r, channel j) within one array of a stage
  static __device__ __forceinline__ int at(int r, int j) { return (j / BOXW) * (C * BOXW) + r * BOXW + (j % BOXW); }
  static constexpr int THREADS = NT + 32;  // + the producer warp
  static constexpr size_t SMEM = (size_t)S * STAGE;
};

// Tile geometry from its ticket.
struct TileGeo {
  long long b;
  int c, nvalid, kvalid;
  long long k0;
};
__device__ __forceinline__ TileGeo tile_geo(const RealParams& p, long long ticket, int K, bool reverse) {
  TileGeo g;
  const int cq = (int)(ticket / p.per_chunk);
  const long long rem = ticket - (long long)cq * p.per_chunk;
  g.c = reverse ? p.chunks - 1 - cq : cq;
  g.b = rem / p.nDB;
  const int db = (int)(rem - g.b * p.nDB);
  g.k0 = (long long)db * K;
  const long long t0 = (long long)g.c * kRealChunk;
  g.nvalid = (int)min((long long)kRealChunk, p.T - t0);
  g.kvalid = (int)min((long long)K, p.D - g.k0);
  return g;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

// Producer warp: takes tickets and stages tiles; a ticket past the last tile ends the stream
// (s_tile = -1 on a stage whose barrier then completes with no copies).
template <typename TA, typename TB, int NT, int S, bool BWD>
__device__ __forceinline__ void produce(const RealParams& p, unsigned char* smem, unsigned long long* full,
                                       unsigned long long* empty, long long* s_tile, unsigned* s_issued) {
  using CF = Cfg<TA, TB, NT, S, BWD>;
  constexpr int C = CF::C, BOXW = CF::BOXW, NBOX = CF::NBOX;
  constexpr unsigned kBatch = 2;  // tickets per claim
  const int lane = threadIdx.x & 31;
  // lane 0 holds the current claim and the next one (requested a claim ahead)
  unsigned cur = 0, nxt = 0, used = 0;
  if (lane == 0) {
    cur = atomicAdd(&p.ls->ticket, kBatch);
    nxt = atomicAdd(&p.ls->ticket, kBatch);
  }
  for (int i = 0;; ++i) {
    const int s = i % S;
    long long ticket = 0;
    if (lane == 0) {
      if (used == kBatch) {
        cur = nxt;
        used = 0;
        nxt = atomicAdd(&p.ls->ticket, kBatch);
      }
      ticket = (long long)cur + used++;
    }
    ticket = __shfl_sync(0xffffffffu, ticket, 0);
    if (i >= S) {
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&empty[s], ((i / S) - 1) & 1, p.max_spin);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) atomicOr(&p.ls->status, kStatusTimeout);
        return;  // consumers stop on their own timeout
      }
    }
    if (ticket >= p.tiles) {
      if (lane == 0) {
        s_tile[s] = -1;
        s_issued[s] += 1;
        mbar_arrive(&full[s]);
      }
      return;
    }
    const TileGeo g = tile_geo(p, ticket, CF::K, BWD);
    const long long row0 = g.b * p.T + (long long)g.c * C;
    unsigned char* st = smem + (size_t)s * CF::STAGE;
    if (p.bulk) {
      if (lane == 0) {
        s_tile[s] = ticket;
        s_issued[s] += 1;
        // whole boxes (zero-filled past the edges), plus the backward's carry row
        const bool hrow = BWD && g.c > 0;
        mbar_arrive_expect_tx(&full[s], (unsigned)(CF::OFF_H + (hrow ? g.kvalid * 4 : 0)));
        if (hrow)
          bulk_copy_g2s(st + CF::OFF_H, p.carry + (g.b * p.chunks + g.c - 1) * p.D + g.k0, (unsigned)(g.kvalid * 4),
                        &full[s]);
        for (int bx = 0; bx < NBOX; ++bx) {
          const int c0 = (int)(g.k0 + bx * BOXW);
          tma_load_2d(st + bx * C * BOXW * (int)sizeof(TA), &p.map_a, c0, (int)row0, &full[s]);
          tma_load_2d(st + CF::OFF_B + bx * C * BOXW * (int)sizeof(TB), &p.map_b, c0, (int)row0, &full[s]);
          if constexpr (BWD)
            tma_load_2d(st + CF::OFF_G + bx * C * BOXW * (int)sizeof(TB), &p.map_g, c0, (int)row0, &full[s]);
        }
      }
    } else {
      // plain staging into the same layout: the warp copies element by element, then arrives
      TA* da = reinterpret_cast<TA*>(st);
      TB* db = reinterpret_cast<TB*>(st + CF::OFF_B);
      TB* dg = reinterpret_cast<TB*>(st + CF::OFF_G);
      const TA* ga = static_cast<const TA*>(p.a);
      const TB* gb = static_cast<const TB*>(p.b);
      const TB* gg = static_cast<const TB*>(p.g);
      for (int row = 0; row < g.nvalid; ++row) {
        const long long base = (row0 + row) * p.D + g.k0;
        for (int jj = lane; jj < g.kvalid; jj += 32) {
          const int o = CF::at(row, jj);
          da[o] = ga[base + jj];
          db[o] = gb[base + jj];
          if constexpr (BWD) dg[o] = gg[base + jj];
        }
      }
      if (BWD && g.c > 0) {
        float* dh = reinterpret_cast<float*>(st + CF::OFF_H);
        const float* gh = p.carry + (g.b * p.chunks + g.c - 1) * p.D + g.k0;
        for (int jj = lane; jj < g.kvalid; jj += 32) dh[jj] = gh[jj];
      }
      __syncwarp();
      if (lane == 0) {
        s_tile[s] = ticket;
        s_issued[s] += 1;
        mbar_arrive(&full[s]);  // release: the warp's shared-memory stores precede it
      }
    }
  }
}

// Carry-in of one channel by decoupled lookback. `pred` is the tile whose status is read first
// (`dist` tickets back; `w_first` its word, already loaded) and `steps_max` the number of tiles
// before this one in its row. Returns the carry (zero after a timed-out wait). (A variant that
// requested the words of four predecessors at once measured slower at every size: the window's
// registers spill in the tile kernels, which hold a whole tile in registers.)
__device__ __forceinline__ float lookback1(const RealParams& p, unsigned epoch, long long pred, long long dist,
                                           int steps_max, int j, int K, unsigned long long w_first) {
  const unsigned tag_incl = make_flag(epoch, kTagInclusive);
  const unsigned tag_agg = make_flag(epoch, kTagAggregate);
  float accA = 1.0f, accB = 0.0f;
  unsigned long long w = w_first;
  for (int step = 1;; ++step) {
    unsigned it = 0;
    for (;;) {
      const unsigned tag = (unsigned)(w >> 32);
      if (tag == tag_incl) return fmaf(accA, __uint_as_float((unsigned)w), accB);
      if (tag == tag_agg) break;
      if (++it >= p.max_spin) {
        atomicOr(&p.ls->status, kStatusTimeout);
        return accB;
      }
      if (it > 8) __nanosleep(it < 64 ? 32 : 128);
      w = ld_relaxed_u64(p.w1 + pred * K + j);
    }
    // aggregate: P in w, Q in the second word (same tag; may become visible a little later)
    unsigned long long q = ld_relaxed_u64(p.w2 + pred * K + j);
    unsigned it2 = 0;
    while ((unsigned)(q >> 32) != tag_agg) {
      if (++it2 >= p.max_spin) {
        atomicOr(&p.ls->status, kStatusTimeout);
        return accB;
      }
      __nanosleep(32);
      q = ld_relaxed_u64(p.w2 + pred * K + j);
    }
    accB = fmaf(accA, __uint_as_float((unsigned)q), accB);
    accA *= __uint_as_float((unsigned)w);
    if (step >= steps_max) return accB;  // unreachable: the first tile of a row always publishes inclusive
    pred -= dist;
    w = ld_relaxed_u64(p.w1 + pred * K + j);
  }
}

// Status of both channels of this thread for tile `t`: aggregate (when the predecessor's
// inclusive was not visible) or inclusive.
__device__ __forceinline__ void publish2(const RealParams& p, long long t, int K, int j, float2 v, unsigned tag) {
  unsigned long long* w = p.w1 + t * K + j;
  st_relaxed_u64(w, make_word(v.x, tag));
  st_relaxed_u64(w + 1, make_word(v.y, tag));
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int c0, int c1, const void* src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(c0),
               "r"(c1), "r"(smem_addr(src))
               : "memory");
}
__device__ __forceinline__ void tma_store_commit_and_wait_read() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Barrier among the NT consumer threads only (the producer warp runs on).
template <int NT>
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"r"(NT) : "memory");
}

// Shared set-up of both kernels: stage barriers (full: the producer's arrival + the tile's bytes;
// empty: one arrival by the consumers' thread 0 once every consumer is done with the stage).
template <int S>
__device__ __forceinline__ void init_stages(unsigned long long* full, unsigned long long* empty, unsigned* s_issued,
                                            unsigned* s_seen) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      s_issued[s] = 0;
      s_seen[s] = 0;
    }
    mbar_init_fence();
  }
  __syncthreads();
}

// End of both kernels: copies still in flight after a timed-out wait complete before the CTA
// exits (bounded), then the launch's epoch bookkeeping.
template <int S>
__device__ __forceinline__ void finish_stages(const RealParams& p, unsigned long long* full, const unsigned* s_issued,
                                              const unsigned* s_seen) {
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s)
      if (s_issued[s] > s_seen[s]) mbar_wait(&full[s], (s_issued[s] - 1) & 1, p.max_spin);
  }
  finish_launch(p.ls);
}

// Consumer wait for the next stage; false ends the consumer loop (end of stream or timeout).
template <int NT, int S>
__device__ __forceinline__ bool next_tile(const RealParams& p, int i, unsigned long long* full, const long long* s_tile,
                                          unsigned* s_seen, long long* t) {
  const int s = i % S;
  if (!mbar_wait(&full[s], (i / S) & 1, p.max_spin)) {
    if ((threadIdx.x & 31) == 0) atomicOr(&p.ls->status, kStatusTimeout);
    return false;
  }
  if (threadIdx.x == 0) s_seen[s] += 1;
  *t = *(volatile const long long*)&s_tile[s];
  return *t >= 0;
}

template <typename TA, typename TB, int NT, int S>
__global__ void __launch_bounds__(NT + 32, 1) real_fwd_kernel(const __grid_constant__ RealParams p) {
  using CF = Cfg<TA, TB, NT, S, false>;
  constexpr int C = CF::C, K = CF::K, BW = CF::BOXW;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ unsigned long long full[S], empty[S];
  __shared__ long long s_tile[S];
  __shared__ unsigned s_issued[S], s_seen[S];
  const int tid = threadIdx.x;
  init_stages<S>(full, empty, s_issued, s_seen);
  const unsigned epoch = *(volatile unsigned*)&p.ls->epoch;
  if (tid >= NT) {
    produce<TA, TB, NT, S, false>(p, smem, full, empty, s_tile, s_issued);
  } else {
    const int j = tid * 2;  // first of this thread's two channels within the tile
    const int e0 = CF::at(0, j);
    const unsigned tag_incl = make_flag(epoch, kTagInclusive);
    long long t;
    for (int i = 0; next_tile<NT, S>(p, i, full, s_tile, s_seen, &t); ++i) {
      const int s = i % S;
      const TileGeo g = tile_geo(p, t, K, false);
      const bool active = j < g.kvalid, two = j + 1 < g.kvalid;
      const long long ch = g.k0 + j;
      // the predecessor's status, requested first so its latency overlaps the summary
      unsigned long long wp0 = 0, wp1 = 0;
      const long long pred = t - p.per_chunk;
      if (g.c > 0) {
        wp0 = ld_relaxed_u64(p.w1 + pred * K + j);
        wp1 = ld_relaxed_u64(p.w1 + pred * K + j + 1);
      }
      unsigned char* st = smem + (size_t)s * CF::STAGE;
      const TA* sa = reinterpret_cast<const TA*>(st) + e0;
      TB* sb = reinterpret_cast<TB*>(st + CF::OFF_B) + e0;
      const bool full_tile = g.nvalid == C;
      // the tile in registers (read from shared memory once), and its map h_out = P h_in + Q
      float2 av[C], bv[C];
      float2 P = make_float2(1.0f, 1.0f), Q = make_float2(0.0f, 0.0f);
      if (full_tile) {
#pragma unroll
        for (int r = 0; r < C; ++r) {
          av[r] = Pair<TA>::ld(sa + r * BW);
          bv[r] = Pair<TB>::ld(sb + r * BW);
        }
      } else {
#pragma unroll
        for (int r = 0; r < C; ++r) {  // padding tokens: a = 1, b = 0
          av[r] = r < g.nvalid ? Pair<TA>::ld(sa + r * BW) : make_float2(1.0f, 1.0f);
          bv[r] = r < g.nvalid ? Pair<TB>::ld(sb + r * BW) : make_float2(0.0f, 0.0f);
        }
      }
#pragma unroll
      for (int r = 0; r < C; ++r) {
        Q = fma2(av[r], Q, bv[r]);
        P = mul2(P, av[r]);
      }
      const bool publish = t != p.inject_unpublished;
      float2 hin = make_float2(0.0f, 0.0f);
      if (g.c > 0) {
        if ((unsigned)(wp0 >> 32) == tag_incl && (unsigned)(wp1 >> 32) == tag_incl) {
          hin = make_float2(__uint_as_float((unsigned)wp0), __uint_as_float((unsigned)wp1));
        } else {
          if (publish) {
            unsigned long long* w2 = p.w2 + t * K + j;
            st_relaxed_u64(w2, make_word(Q.x, make_flag(epoch, kTagAggregate)));
            st_relaxed_u64(w2 + 1, make_word(Q.y, make_flag(epoch, kTagAggregate)));
            publish2(p, t, K, j, P, make_flag(epoch, kTagAggregate));
          }
          hin.x = lookback1(p, epoch, pred, p.per_chunk, g.c, j, K, wp0);
          hin.y = lookback1(p, epoch, pred, p.per_chunk, g.c, j + 1, K, wp1);
        }
      }
      const float2 hout = fma2(P, hin, Q);
      if (publish) publish2(p, t, K, j, hout, tag_incl);
      if (active) {
        float* cp = p.carry + (g.b * p.chunks + g.c) * p.D + ch;
        cp[0] = hout.x;
        if (two) cp[1] = hout.y;
        if (g.c == p.chunks - 1 && p.last != nullptr) {
          p.last[g.b * p.D + ch] = hout.x;
          if (two) p.last[g.b * p.D + ch + 1] = hout.y;
        }
      }
      const long long row0 = g.b * p.T + (long long)g.c * C;
      const bool tma_out = full_tile && p.bulk;
      float2 h = hin;
      if (tma_out) {
        // the states replace b in shared memory; one TMA store per box writes them out
#pragma unroll
        for (int r = 0; r < C; ++r) {
          h = fma2(av[r], h, bv[r]);
          Pair<TB>::st(sb + r * BW, h);
        }
        fence_proxy_async_smem();
      } else if (active) {
        TB* po = static_cast<TB*>(p.out) + row0 * p.D + ch;
#pragma unroll
        for (int r = 0; r < C; ++r) {
          if (r < g.nvalid) {
            h = fma2(av[r], h, bv[r]);
            const long long o = (long long)r * p.D;
            Pair<TB>::st1(po + o, h.x);
            if (two) Pair<TB>::st1(po + o + 1, h.y);
          }
        }
      }
      consumers_sync<NT>();
      if (tid == 0) {
        if (tma_out) {
#pragma unroll
          for (int bx = 0; bx < CF::NBOX; ++bx)
            tma_store_2d(&p.map_o, (int)(g.k0 + bx * BW), (int)row0, st + CF::OFF_B + bx * C * BW * (int)sizeof(TB));
          tma_store_commit_and_wait_read();
        }
        mbar_arrive(&empty[s]);
      }
    }
  }
  finish_stages<S>(p, full, s_issued, s_seen);
}

template <typename TA, typename TB, int NT, int S>
__global__ void __launch_bounds__(NT + 32, 1) real_bwd_kernel(const __grid_constant__ RealParams p) {
  using CF = Cfg<TA, TB, NT, S, true>;
  constexpr int C = CF::C, K = CF::K, BW = CF::BOXW;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ unsigned long long full[S], empty[S];
  __shared__ long long s_tile[S];
  __shared__ unsigned s_issued[S], s_seen[S];
  const int tid = threadIdx.x;
  init_stages<S>(full, empty, s_issued, s_seen);
  const unsigned epoch = *(volatile unsigned*)&p.ls->epoch;
  if (tid >= NT) {
    produce<TA, TB, NT, S, true>(p, smem, full, empty, s_tile, s_issued);
  } else {
    const int j = tid * 2;
    const int e0 = CF::at(0, j);
    const unsigned tag_incl = make_flag(epoch, kTagInclusive);
    long long t;
    for (int i = 0; next_tile<NT, S>(p, i, full, s_tile, s_seen, &t); ++i) {
      const int s = i % S;
      const TileGeo g = tile_geo(p, t, K, true);
      const bool active = j < g.kvalid, two = j + 1 < g.kvalid;
      const long long ch = g.k0 + j;
      const bool last_chunk = g.c == p.chunks - 1;
      unsigned long long wp0 = 0, wp1 = 0;
      const long long succ = t - p.per_chunk;  // the chunk to the right (processed first)
      if (!last_chunk) {
        wp0 = ld_relaxed_u64(p.w1 + succ * K + j);
        wp1 = ld_relaxed_u64(p.w1 + succ * K + j + 1);
      }
      unsigned char* st = smem + (size_t)s * CF::STAGE;
      TA* sa = reinterpret_cast<TA*>(st) + e0;
      const TB* sb = reinterpret_cast<const TB*>(st + CF::OFF_B) + e0;
      TB* sg = reinterpret_cast<TB*>(st + CF::OFF_G) + e0;
      // the state entering the chunk, staged with the tile (channels past kvalid: unused)
      const float2 hin = g.c > 0 ? *reinterpret_cast<const float2*>(st + CF::OFF_H + j * 4) : make_float2(0.0f, 0.0f);
      const bool full_tile = g.nvalid == C;
      // a and the replayed states in registers (h[r]: after token r; padding tokens a = 1, b = 0)
      float2 av[C], h[C];
      {
        float2 hh = hin;
#pragma unroll
        for (int r = 0; r < C; ++r) {
          const bool v = full_tile || r < g.nvalid;
          av[r] = v ? Pair<TA>::ld(sa + r * BW) : make_float2(1.0f, 1.0f);
          const float2 bb = v ? Pair<TB>::ld(sb + r * BW) : make_float2(0.0f, 0.0f);
          hh = fma2(av[r], hh, bb);
          h[r] = hh;
        }
      }
      // the chunk's reverse map: kappa_out = P kappa_in + Qr (kappa = a lambda entering / leaving)
      float2 P = make_float2(1.0f, 1.0f), Qr = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int r = C - 1; r >= 0; --r) {
        const float2 gg = (full_tile || r < g.nvalid) ? Pair<TB>::ld(sg + r * BW) : make_float2(0.0f, 0.0f);
        Qr = mul2(add2(Qr, gg), av[r]);
        P = mul2(P, av[r]);
      }
      float2 kin = make_float2(0.0f, 0.0f);
      if (!last_chunk) {
        if ((unsigned)(wp0 >> 32) == tag_incl && (unsigned)(wp1 >> 32) == tag_incl) {
          kin = make_float2(__uint_as_float((unsigned)wp0), __uint_as_float((unsigned)wp1));
        } else {
          unsigned long long* w2 = p.w2 + t * K + j;
          st_relaxed_u64(w2, make_word(Qr.x, make_flag(epoch, kTagAggregate)));
          st_relaxed_u64(w2 + 1, make_word(Qr.y, make_flag(epoch, kTagAggregate)));
          publish2(p, t, K, j, P, make_flag(epoch, kTagAggregate));
          const int steps = p.chunks - 1 - g.c;
          kin.x = lookback1(p, epoch, succ, p.per_chunk, steps, j, K, wp0);
          kin.y = lookback1(p, epoch, succ, p.per_chunk, steps, j + 1, K, wp1);
        }
      }
      publish2(p, t, K, j, fma2(P, kin, Qr), tag_incl);
      const long long row0 = g.b * p.T + (long long)g.c * C;
      const bool tma_out = full_tile && p.bulk;
      float2 lam = kin;
      if (tma_out) {
        // grad_a replaces a and grad_b replaces grad_out in shared memory (each thread reads its
        // own element before overwriting it); one TMA store per box and array writes them out
#pragma unroll
        for (int r = C - 1; r >= 0; --r) {
          lam = add2(lam, Pair<TB>::ld(sg + r * BW));
          Pair<TA>::st(sa + r * BW, mul2(lam, r > 0 ? h[r - 1] : hin));
          Pair<TB>::st(sg + r * BW, lam);
          lam = mul2(lam, av[r]);
        }
        fence_proxy_async_smem();
      } else if (active) {
        TA* pga = static_cast<TA*>(p.out) + row0 * p.D + ch;
        TB* pgb = static_cast<TB*>(p.out2) + row0 * p.D + ch;
#pragma unroll
        for (int r = C - 1; r >= 0; --r) {
          if (r < g.nvalid) {
            lam = add2(lam, Pair<TB>::ld(sg + r * BW));
            const float2 ga = mul2(lam, r > 0 ? h[r - 1] : hin);
            const long long o = (long long)r * p.D;
            Pair<TA>::st1(pga + o, ga.x);
            Pair<TB>::st1(pgb + o, lam.x);
            if (two) {
              Pair<TA>::st1(pga + o + 1, ga.y);
              Pair<TB>::st1(pgb + o + 1, lam.y);
            }
            lam = mul2(lam, av[r]);
          }
        }
      }
      consumers_sync<NT>();
      if (tid == 0) {
        if (tma_out) {
#pragma unroll
          for (int bx = 0; bx < CF::NBOX; ++bx) {
            const int c0 = (int)(g.k0 + bx * BW);
            tma_store_2d(&p.map_o, c0, (int)row0, st + bx * C * BW * (int)sizeof(TA));
            tma_store_2d(&p.map_o2, c0, (int)row0, st + CF::OFF_G + bx * C * BW * (int)sizeof(TB));
          }
          tma_store_commit_and_wait_read();
        }
        mbar_arrive(&empty[s]);
      }
    }
  }
  finish_stages<S>(p, full, s_issued, s_seen);
}

// ------------------------------------------------------------------------------------ host
// Consumer threads per CTA (NT; a tile is K = 2 NT channels of 32 tokens) and the shared-memory
// budget per CTA, from which the stage count S follows (2..6). Two shapes of tile:
//  * wide (K = 512 forward): one CTA per SM, for problems with many tiles per chunk;
//  * narrow (K = 128): several CTAs per SM, for problems with few channels, where wide tiles
//    would leave too few tiles per chunk and make every lookback walk back over several chunks.
// Build-time tunables (-D...) for measurement; the defaults are the measured best.
#ifndef SPARC_REAL_NT_FWD
#define SPARC_REAL_NT_FWD 256
#endif
#ifndef SPARC_REAL_NT_BWD
#define SPARC_REAL_NT_BWD 256
#endif
#ifndef SPARC_REAL_NT_NARROW
#define SPARC_REAL_NT_NARROW 64
#endif
#ifndef SPARC_REAL_WIDE_SMEM
#define SPARC_REAL_WIDE_SMEM (200 * 1024)
#endif
#ifndef SPARC_REAL_NARROW_SMEM
#define SPARC_REAL_NARROW_SMEM (72 * 1024)
#endif
constexpr int kRealMaxSmem = 225 * 1024;  // dynamic shared memory a CTA may opt in to (2 stages at least)
template <typename TA, typename TB, bool BWD, bool WIDE>
struct Choice {
  static constexpr int NT0 = WIDE ? (BWD ? SPARC_REAL_NT_BWD : SPARC_REAL_NT_FWD) : SPARC_REAL_NT_NARROW;
  // halve the tile until two stages fit (float32 arrays on a 512-channel tile do not)
  static constexpr int NT1 = 2 * Cfg<TA, TB, NT0, 2, BWD>::STAGE <= kRealMaxSmem ? NT0 : NT0 / 2;
  static constexpr int NT = 2 * Cfg<TA, TB, NT1, 2, BWD>::STAGE <= kRealMaxSmem ? NT1 : NT1 / 2;
  static constexpr int STAGE = Cfg<TA, TB, NT, 2, BWD>::STAGE;
  static constexpr int S0 = (WIDE ? SPARC_REAL_WIDE_SMEM : SPARC_REAL_NARROW_SMEM) / STAGE;
  static constexpr int S = S0 < 2 ? 2 : S0 > 6 ? 6 : S0;
};
constexpr int kRealMaxK = 512;  // the widest tile of any choice (workspace sizing)
static_assert(2 * SPARC_REAL_NT_FWD <= kRealMaxK && 2 * SPARC_REAL_NT_BWD <= kRealMaxK &&
              2 * SPARC_REAL_NT_NARROW <= kRealMaxK, "tiles of at most 512 channels");

template <typename TA, typename TB, bool BWD, bool WIDE>
static const void* kernel_of() {
  using CH = Choice<TA, TB, BWD, WIDE>;
  if constexpr (BWD) return (const void*)real_bwd_kernel<TA, TB, CH::NT, CH::S>;
  else return (const void*)real_fwd_kernel<TA, TB, CH::NT, CH::S>;
}

struct Launch {
  const void* kernel;
  int threads, K, boxw;
  size_t smem;
};

template <typename TA, typename TB, bool BWD, bool WIDE>
static Launch launch_of() {
  using CH = Choice<TA, TB, BWD, WIDE>;
  using CF = Cfg<TA, TB, CH::NT, CH::S, BWD>;
  return Launch{kernel_of<TA, TB, BWD, WIDE>(), CF::THREADS, CF::K, CF::BOXW, CF::SMEM};
}

template <bool WIDE>
static Launch pick_shape(int a_dtype, int b_dtype, bool bwd) {
  const bool af = a_dtype == SPARC_DTYPE_F32, bf = b_dtype == SPARC_DTYPE_F32;
  if (bwd) {
    if (af && bf) return launch_of<float, float, true, WIDE>();
    if (af) return launch_of<float, __nv_bfloat16, true, WIDE>();
    if (bf) return launch_of<__nv_bfloat16, float, true, WIDE>();
    return launch_of<__nv_bfloat16, __nv_bfloat16, true, WIDE>();
  }
  if (af && bf) return launch_of<float, float, false, WIDE>();
  if (af) return launch_of<float, __nv_bfloat16, false, WIDE>();
  if (bf) return launch_of<__nv_bfloat16, float, false, WIDE>();
  return launch_of<__nv_bfloat16, __nv_bfloat16, false, WIDE>();
}

// Wide tiles when a chunk has at least two tiles per SM of them, else narrow.
static Launch pick(int a_dtype, int b_dtype, bool bwd, long long B, long long D, int sms) {
  const Launch w = pick_shape<true>(a_dtype, b_dtype, bwd);
  if (B * ((D + w.K - 1) / w.K) >= 2LL * sms) return w;
  return pick_shape<false>(a_dtype, b_dtype, bwd);
}

static bool valid_dtype(int d) { return d == SPARC_DTYPE_F32 || d == SPARC_DTYPE_BF16; }
static int esize(int d) { return d == SPARC_DTYPE_F32 ? 4 : 2; }

// Opt-in to the launch's shared memory once per (device, kernel) and return the grid: one CTA
// per SM (or fewer, if the tiles are fewer).
static int prepare_grid(const Launch& L, long long tiles) {
  static std::mutex mu;
  static const void* done[64][8] = {};
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) { cudaGetLastError(); return 0; }
  {
    std::lock_guard<std::mutex> lock(mu);
    bool set = false;
    int slot = -1;
    for (int k = 0; k < 8; ++k) {
      if (done[dev][k] == L.kernel) { set = true; break; }
      if (done[dev][k] == nullptr && slot < 0) slot = k;
    }
    if (!set) {
      if (cudaFuncSetAttribute(L.kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
      }
      if (slot >= 0) done[dev][slot] = L.kernel;
    }
  }
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) { cudaGetLastError(); return 0; }
  int per = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, L.kernel, L.threads, L.smem) != cudaSuccess || per <= 0) {
    cudaGetLastError();
    return 0;
  }
  return (int)std::min<long long>((long long)per * sms, tiles);
}

struct RealGeom {
  int chunks, nDB;
  long long tiles, per_chunk;
};

static int real_geom(long long B, long long T, long long D, int K, RealGeom* g) {
  if (B <= 0 || T <= 0 || D <= 0) return fail(SPARC_ERR_SHAPE, "batch, length and channels must be positive");
  g->chunks = (int)((T + kRealChunk - 1) / kRealChunk);
  g->nDB = (int)((D + K - 1) / K);
  g->per_chunk = B * (long long)g->nDB;
  g->tiles = g->per_chunk * g->chunks;
  if (g->tiles >= (1LL << 31) || T >= (1LL << 40) || D >= (1LL << 31))
    return fail(SPARC_ERR_SHAPE, "too many tiles");
  return SPARC_OK;
}

// Workspace: launch state, then w1 and w2 [tiles, K] 64-bit words each, sized for the widest
// tile so one size serves every dtype pair and direction.
static size_t real_ws_total(long long B, long long T, long long D) {
  const long long chunks = (T + kRealChunk - 1) / kRealChunk;
  const long long Dp = (D + kRealMaxK - 1) / kRealMaxK * kRealMaxK;
  const size_t words = (size_t)B * chunks * Dp;
  return 256 + 2 * ((words * 8 + 255) & ~size_t(255));
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
static PFN_cuTensorMapEncodeTiled_v12000 real_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    } else {
      cudaGetLastError();
    }
  });
  return fn;
}

// [rows, D] row-major as a 2-D map with a {boxw, 32} box (no swizzle: the stage keeps rows of
// boxw elements), zero fill past the edges.
static bool real_map(CUtensorMap* map, const void* base, int dtype, long long rows, long long D, int boxw) {
  const PFN_cuTensorMapEncodeTiled_v12000 enc = real_map_encoder();
  if (enc == nullptr) return false;
  const cuuint64_t es = (cuuint64_t)esize(dtype);
  const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)D * es};
  const cuuint32_t box[2] = {(cuuint32_t)boxw, (cuuint32_t)kRealChunk};
  const cuuint32_t estride[2] = {1, 1};
  return enc(map, dtype == SPARC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
             const_cast<void*>(base), dims, strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int real_launch(RealParams& p, const void* ws, size_t ws_bytes, int a_dtype, int b_dtype, bool bwd,
                       cudaStream_t s) {
  if (!valid_dtype(a_dtype) || !valid_dtype(b_dtype)) return fail(SPARC_ERR_DTYPE, "unsupported dtype");
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    return fail(SPARC_ERR_LAUNCH, "no current CUDA device");
  }
  const Launch L = pick(a_dtype, b_dtype, bwd, p.B, p.D, sms);
  RealGeom g;
  int rc = real_geom(p.B, p.T, p.D, L.K, &g);
  if (rc != SPARC_OK) return rc;
  const size_t need = real_ws_total(p.B, p.T, p.D);
  if (ws == nullptr || ws_bytes < need) return fail(SPARC_ERR_WORKSPACE, "workspace too small");
  char* w = static_cast<char*>(const_cast<void*>(ws));
  const size_t half = (need - 256) / 2;
  p.ls = reinterpret_cast<LaunchState*>(w);
  p.w1 = reinterpret_cast<unsigned long long*>(w + 256);
  p.w2 = reinterpret_cast<unsigned long long*>(w + 256 + half);
  p.chunks = g.chunks;
  p.nDB = g.nDB;
  p.tiles = g.tiles;
  p.per_chunk = g.per_chunk;
  // tiles by TMA tensor copies when every row is whole 16-byte units at 16-byte aligned addresses
  // (the maps' stride rule) and the row coordinate fits a 32-bit TMA coordinate
  const int sa = esize(a_dtype), sb = esize(b_dtype);
  const long long rows = p.B * p.T;
  bool bulk = (p.D * sa) % 16 == 0 && (p.D * sb) % 16 == 0 && aligned16(p.a) && aligned16(p.b) &&
              rows + kRealChunk < (1LL << 31);
  if (bwd) bulk = bulk && aligned16(p.g) && aligned16(p.out) && aligned16(p.out2) && aligned16(p.carry);
  else bulk = bulk && aligned16(p.out);
  if (bulk) {
    bulk = real_map(&p.map_a, p.a, a_dtype, rows, p.D, L.boxw) && real_map(&p.map_b, p.b, b_dtype, rows, p.D, L.boxw);
    if (bwd)
      bulk = bulk && real_map(&p.map_g, p.g, b_dtype, rows, p.D, L.boxw) &&
             real_map(&p.map_o, p.out, a_dtype, rows, p.D, L.boxw) && real_map(&p.map_o2, p.out2, b_dtype, rows, p.D, L.boxw);
    else
      bulk = bulk && real_map(&p.map_o, p.out, b_dtype, rows, p.D, L.boxw);
  }
  p.bulk = bulk ? 1 : 0;
  const int grid = prepare_grid(L, g.tiles);
  if (grid <= 0) return fail(SPARC_ERR_LAUNCH, "shared-memory opt-in or occupancy query failed");
  TimedLaunch tl(bwd ? kTimeRealBwd : kTimeRealFwd, s);
  void* args[] = {&p};
  const cudaError_t e = cudaLaunchKernel(L.kernel, dim3(grid), dim3(L.threads), args, L.smem, s);
  return e == cudaSuccess ? SPARC_OK : fail(SPARC_ERR_LAUNCH, cudaGetErrorString(e));
}

}  // namespace sparc

using namespace sparc;

extern "C" {

long long sparc_real_chunk_tokens(void) { return kRealChunk; }

long long sparc_real_carry_chunks(long long length) { return (length + kRealChunk - 1) / kRealChunk; }

size_t sparc_real_workspace_bytes(long long batch, long long length, long long channels, int dtype) {
  if (batch <= 0 || length <= 0 || channels <= 0) { fail(SPARC_ERR_SHAPE, "batch, length and channels must be positive"); return 0; }
  if (!valid_dtype(dtype)) { fail(SPARC_ERR_DTYPE, "unsupported dtype"); return 0; }
  return real_ws_total(batch, length, channels);
}

int sparc_real_scan_forward(const SparcRealFwdArgs* a, void* stream) {
  NvtxRange nvtx(__func__);
  if (a == nullptr) return fail(SPARC_ERR_ARG, "null args");
  if (!a->a || !a->b || !a->out || !a->carry) return fail(SPARC_ERR_ARG, "null tensor pointer");
  if (a->batch <= 0 || a->length <= 0 || a->channels <= 0)
    return fail(SPARC_ERR_SHAPE, "batch, length and channels must be positive");
  if (!valid_dtype(a->dtype) || !valid_dtype(a->a_dtype)) return fail(SPARC_ERR_DTYPE, "unsupported dtype");
  RealParams p{};
  p.a = a->a;
  p.b = a->b;
  p.out = a->out;
  p.last = a->last;
  p.carry = a->carry;
  p.B = a->batch;
  p.T = a->length;
  p.D = a->channels;
  p.max_spin = a->max_spin ? a->max_spin : (1u << 20);
  p.inject_unpublished = a->inject_enable ? a->inject_tile : -1;
  return real_launch(p, a->workspace, a->workspace_bytes, a->a_dtype, a->dtype, false,
                     static_cast<cudaStream_t>(stream));
}

int sparc_real_scan_backward(const SparcRealBwdArgs* a, void* stream) {
  NvtxRange nvtx(__func__);
  if (a == nullptr) return fail(SPARC_ERR_ARG, "null args");
  if (!a->a || !a->b || !a->grad_out || !a->carry || !a->grad_a || !a->grad_b)
    return fail(SPARC_ERR_ARG, "null tensor pointer");
  if (a->batch <= 0 || a->length <= 0 || a->channels <= 0)
    return fail(SPARC_ERR_SHAPE, "batch, length and channels must be positive");
  if (!valid_dtype(a->dtype) || !valid_dtype(a->a_dtype)) return fail(SPARC_ERR_DTYPE, "unsupported dtype");
  RealParams p{};
  p.a = a->a;
  p.b = a->b;
  p.g = a->grad_out;
  p.out = a->grad_a;
  p.out2 = a->grad_b;
  p.carry = const_cast<float*>(a->carry);
  p.B = a->batch;
  p.T = a->length;
  p.D = a->channels;
  p.max_spin = a->max_spin ? a->max_spin : (1u << 20);
  p.inject_unpublished = -1;
  return real_launch(p, a->workspace, a->workspace_bytes, a->a_dtype, a->dtype, true,
                     static_cast<cudaStream_t>(stream));
}

}  // extern "C"
