// SPARC mixer forward kernels (included by mixer.cu, which holds the shared helpers and the
// carry scan). The forward is three launches:
//
//   mixer_fwd_summary_kernel   per tile (batch row b, chunk of C tokens, all M modes): the
//                              token controls (projection of x onto the two controller
//                              directions, reduced over all modes: warp transpose-reduce ->
//                              shared memory -> distributed shared memory across the cluster of
//                              G CTAs that share the tile), saved per token for the replay and
//                              the backward; then the chunk's aggregate affine map
//                              h_out = P h_in + Q per mode (P = prod a_t, Q = the local scan).
//   mixer_carry_scan_kernel    (mixer.cu) the inclusive chunk states from the aggregates.
//   mixer_fwd_replay_kernel    per tile again: from the carried-in state, h_t = a_t h_{t-1} + b_t
//                              and y = relu([Re h, Im h]).
//
// Both tile kernels are persistent with a static schedule (tile k, k + n, k + 2n, ... for the
// k-th of n CTAs or clusters): tiles do not depend on each other, so nothing waits on another
// CTA. x tiles (and the replay's controls and carried-in states) arrive in shared memory by
// TMA bulk copies on an mbarrier, double-buffered so the next tile's copy overlaps this tile's
// arithmetic. CTA g of a tile owns modes [g*256, g*256+256), two adjacent modes per thread.

// (included inside namespace sparc)

constexpr int kFwdThreads = 128;
constexpr int kFwdModes = 2 * kFwdThreads;  // modes per CTA

template <typename TIO, int C>
struct SumSmem {
  TIO x[2][C][2][kFwdModes];  // [buffer][token][re|im][mode]
  TokenCtl ctl[C];
  float part_all[2][8][3 * C];  // every cluster CTA's projection / sum-of-squares partials (pushed
                                // by the peers), by tile parity
  float warp_part[kFwdThreads / 32][3 * C];
  unsigned long long bar[2];
  unsigned long long red[2];    // completes when all G CTAs' partials of a tile have arrived
};

template <typename TIO, int C>
struct RepSmem {
  TIO x[2][C][2][kFwdModes];
  TokenCtl ctl[2][C];
  unsigned long long bar[2];
};

struct FwdParams {
  CUtensorMap map_x;    // x as [B*T rows][re|im][M], box {256, 2, C} (when use_tma)
  const void* x;
  void* y;
  void* states;         // [B*T, W] every token's state [Re | Im] (dtype) for the backward, or null
  MixerParamPtrs pp;
  const float* h0_r;
  const float* h0_i;
  TokenCtl* ctl;        // [B, T] token controls (written by the summary)
  const unsigned char* reset;  // [B, T] 1 where a segment reset zeroes the transition, or null
  const float* norm_w;  // [W] RMSNorm weight of a block (kBlock kernels), else null
  float norm_eps;
  unsigned* mask;       // [B*T, mask_words] relu bits of the block's mixer output (kBlock)
  int mask_words;       // 16 per CTA of 256 modes: four words per 64 modes (store_relu_bits)
  const float2* carry;  // [B, chunks, M] inclusive chunk states (replay input)
  float4* agg;          // [B, chunks, Mp] chunk aggregates (P, Q)
  const float2* proj_in;  // [B*T] controller projections (p0, p1), bias included (kModeProj), or
                          // the controls (delta, eta) themselves (kModeScan)
  int content_linear;     // kModeProj: the content is u itself instead of tanh(u)
  void* y_im;             // kModeScan: Im h [B*T, M] (y then holds Re h [B*T, M]), or null
  LaunchState* ls;
  long long B, T;
  int W, M, Mp, chunks;
  long long tiles;
  unsigned max_spin;
  int use_tma;
};

template <typename TIO> struct Pair;
template <> struct Pair<float> {
  static __device__ __forceinline__ float2 load(const float* p) { return *reinterpret_cast<const float2*>(p); }
  static __device__ __forceinline__ void store(float* p, float a, float b) {
    *reinterpret_cast<float2*>(p) = make_float2(a, b);
  }
};
template <> struct Pair<__nv_bfloat16> {
  static __device__ __forceinline__ float2 load(const __nv_bfloat16* p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float a, float b) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
  }
};

// Store the relu'd (kRelu) or raw pair of states of modes (m, m+1) for one token row.
template <typename TIO, bool kVec, bool kRelu = true>
__device__ __forceinline__ void store_y_pair(TIO* row, int M, int m, bool a0, bool a1, float2 h0, float2 h1) {
  if constexpr (!kRelu) {
    if (kVec && a1) {
      Pair<TIO>::store(row + m, h0.x, h1.x);
      Pair<TIO>::store(row + M + m, h0.y, h1.y);
      return;
    }
    if (a0) {
      Io<TIO>::store(row + m, h0.x);
      Io<TIO>::store(row + M + m, h0.y);
    }
    if (a1) {
      Io<TIO>::store(row + m + 1, h1.x);
      Io<TIO>::store(row + M + m + 1, h1.y);
    }
    return;
  }
  if (kVec) {
    if (a1) {
      Pair<TIO>::store(row + m, fmaxf(h0.x, 0.0f), fmaxf(h1.x, 0.0f));
      Pair<TIO>::store(row + M + m, fmaxf(h0.y, 0.0f), fmaxf(h1.y, 0.0f));
      return;
    }
  }
  if (a0) {
    Io<TIO>::store(row + m, fmaxf(h0.x, 0.0f));
    Io<TIO>::store(row + M + m, fmaxf(h0.y, 0.0f));
  }
  if (a1) {
    Io<TIO>::store(row + m + 1, fmaxf(h1.x, 0.0f));
    Io<TIO>::store(row + M + m + 1, fmaxf(h1.y, 0.0f));
  }
}

// Block output x + relu(h) for the pair of modes (m, m+1) of one token row.
template <typename TIO, bool kVec>
__device__ __forceinline__ void store_sum_pair(TIO* row, int M, int m, bool a0, bool a1, float2 xr, float2 xi,
                                               const Cx2& h) {
  const float r0 = xr.x + fmaxf(h.re.x, 0.0f), r1 = xr.y + fmaxf(h.re.y, 0.0f);
  const float i0 = xi.x + fmaxf(h.im.x, 0.0f), i1 = xi.y + fmaxf(h.im.y, 0.0f);
  if (kVec && a1) {
    Pair<TIO>::store(row + m, r0, r1);
    Pair<TIO>::store(row + M + m, i0, i1);
    return;
  }
  if (a0) {
    Io<TIO>::store(row + m, r0);
    Io<TIO>::store(row + M + m, i0);
  }
  if (a1) {
    Io<TIO>::store(row + m + 1, r1);
    Io<TIO>::store(row + M + m + 1, i1);
  }
}

// Relu bits of one token for the warp's 64 modes (lane l owns modes 2l, 2l+1): four words,
// [real of even modes, real of odd modes, imaginary of even, imaginary of odd], bit l each.
__device__ __forceinline__ void store_relu_bits(unsigned* dst, const Cx2& h, int lane) {
  const unsigned w0 = __ballot_sync(0xffffffffu, h.re.x > 0.0f);
  const unsigned w1 = __ballot_sync(0xffffffffu, h.re.y > 0.0f);
  const unsigned w2 = __ballot_sync(0xffffffffu, h.im.x > 0.0f);
  const unsigned w3 = __ballot_sync(0xffffffffu, h.im.y > 0.0f);
  if (lane == 0) *reinterpret_cast<uint4*>(dst) = make_uint4(w0, w1, w2, w3);
}

// Tile geometry shared by all tile kernels: tile i covers row b = i % B, chunk c = i / B (tile
// counts stay below 2^31, so the division is 32-bit).
struct TileRef {
  long long b;
  int c;
  long long t0;
  int nvalid;
};
__device__ __forceinline__ TileRef tile_ref(long long i, long long B, long long T, int C) {
  TileRef r;
  const unsigned ui = (unsigned)i, ub = (unsigned)B;
  const unsigned c = ui / ub;
  r.c = (int)c;
  r.b = (long long)(ui - c * ub);
  r.t0 = (long long)r.c * C;
  r.nvalid = (int)(T - r.t0 < C ? T - r.t0 : C);
  return r;
}

// The same rows by plain loads spread over the CTA (shapes that are not 16-byte aligned).
template <typename TIO, int NM>
__device__ __forceinline__ void load_act_rows(const TIO* src, int W, int M, int mbase, int nvalid,
                                              TIO (*dst)[2][NM], int nthreads) {
  const int ncols = min(NM, M - mbase);
  const TIO* s = src + mbase;
  for (int i = threadIdx.x; i < nvalid * 2 * ncols; i += nthreads) {
    const int t = i / (2 * ncols), r = i - t * 2 * ncols, half = r / ncols, mm = r - half * ncols;
    dst[t][half][mm] = s[(long long)t * W + half * M + mm];
  }
}

// Bytes of one activation box (the tensor-map copy always moves the whole box; columns past M
// and rows past the tensor arrive as zeros).
template <typename TIO, int C, int NM>
__host__ __device__ constexpr unsigned act_box_bytes() {
  return (unsigned)(NM * 2 * C * sizeof(TIO));
}

// ------------------------------------------------------------------------------ summary
template <typename TIO, int C, bool kFast, int kMode>
__global__ void __launch_bounds__(kFwdThreads) mixer_fwd_summary_kernel(const __grid_constant__ FwdParams p) {
  constexpr int NW = kFwdThreads / 32;
  constexpr bool kBlock = kMode == kModeBlock, kProj = proj_like<kMode>(), kScan = kMode == kModeScan;
  cg::cluster_group cluster = cg::this_cluster();
  const int g = (int)cluster.block_rank();
  const int G = (int)cluster.num_blocks();
  const int tid = threadIdx.x;
  const int M = p.M, W = p.W;
  const int mbase = g * kFwdModes;
  const int m0 = mbase + 2 * tid;  // this thread's modes: m0, m0 + 1
  const bool act0 = m0 < M, act1 = m0 + 1 < M;
  const long long B = p.B, T = p.T;
  const long long k0 = blockIdx.y, nk = gridDim.y;
  pdl_wait();  // the first launch of the forward: parameters may have just been updated

  extern __shared__ __align__(128) unsigned char smem_raw[];
  SumSmem<TIO, C>& S = *reinterpret_cast<SumSmem<TIO, C>*>(smem_raw);

  ModeConst2 mc = pair_modes(load_mode(p.pp, m0, M, act0), load_mode(p.pp, m0 + 1, M, act1));
  if constexpr (kBlock) load_norm_weight(mc, p.norm_w, m0, M, act0, act1);
  const float bias0 = kProj ? 0.0f : p.pp.phase_dir[W], bias1 = kProj ? 0.0f : p.pp.radial_dir[W];
  const bool lin = kProj && p.content_linear != 0;
  // projection directions seen by raw x: D w (the norm's weight), scaled by r after the reduction
  const float2 d0r = mul2(mc.d0r, mc.wre), d0i = mul2(mc.d0i, mc.wim);
  const float2 d1r = mul2(mc.d1r, mc.wre), d1i = mul2(mc.d1i, mc.wim);

  // columns past M are never copied and must read as zeros
  {
    unsigned* xs = reinterpret_cast<unsigned*>(&S.x[0][0][0][0]);
    for (int i = tid; i < (int)(sizeof(S.x) / 4); i += kFwdThreads) xs[i] = 0u;
  }
  constexpr int kVals = kBlock ? 3 * C : 2 * C;  // reduced per-token values
  const unsigned red_bytes = (unsigned)(G * kVals) * 4u;
  if (tid == 0) {
    mbar_init(&S.bar[0], 1);
    mbar_init(&S.bar[1], 1);
    mbar_init(&S.red[0], 1);
    mbar_init(&S.red[1], 1);
    mbar_init_fence();
    if (!kProj && G > 1) {  // armed for tiles 0 and 1 before any peer can push
      mbar_arrive_expect_tx(&S.red[0], red_bytes);
      mbar_arrive_expect_tx(&S.red[1], red_bytes);
    }
  }
  if (G > 1) cluster.sync();  // every CTA's barriers are initialised and armed
  else __syncthreads();

  auto issue = [&](long long i, int buf) {
    const TileRef r = tile_ref(i, B, T, C);
    const TIO* src = static_cast<const TIO*>(p.x) + (r.b * T + r.t0) * W;
    if (p.use_tma) {
      if (tid == 0) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&S.bar[buf], act_box_bytes<TIO, C, kFwdModes>());
        tma_load_3d(&S.x[buf][0][0][0], &p.map_x, mbase, 0, (int)(r.b * T + r.t0), &S.bar[buf]);
      }
    } else {
      load_act_rows<TIO, kFwdModes>(src, W, M, mbase, r.nvalid, S.x[buf], kFwdThreads);
    }
  };
  if (k0 < p.tiles) issue(k0, 0);
  bool timed_out = false;

  for (long long n = 0;; ++n) {
    const long long i = k0 + n * nk;
    if (i >= p.tiles) break;
    const int buf = (int)(n & 1);
    if (i + nk < p.tiles) issue(i + nk, buf ^ 1);
    const TileRef r = tile_ref(i, B, T, C);
    if (p.use_tma) {
      if (!mbar_wait(&S.bar[buf], (unsigned)((n >> 1) & 1), p.max_spin << 4)) timed_out = true;
    } else {
      __syncthreads();
    }
    const TIO(*xt)[2][kFwdModes] = S.x[buf];

    // control projections (and, in a block, the sum of squares for the norm): per-thread
    // partials over its 4 columns, reduced over the cluster; given per token in projection mode
    float p0 = 0.0f, p1 = 0.0f, rs = 1.0f;  // (threads tid < C: token tid's values)
    if constexpr (kProj) {
      if (tid < r.nvalid) {
        const float2 pj = p.proj_in[r.b * T + r.t0 + tid];
        p0 = pj.x;
        p1 = pj.y;
      }
    } else {
      const int lane = tid & 31, warp = tid >> 5;
      float v[2 * C];
      float vs[C];
#pragma unroll
      for (int t = 0; t < C; ++t) {
        const float2 xr = Pair<TIO>::load(&xt[t][0][2 * tid]);
        const float2 xi = Pair<TIO>::load(&xt[t][1][2 * tid]);
        const float2 v0 = fma2(xr, d0r, mul2(xi, d0i));
        const float2 v1 = fma2(xr, d1r, mul2(xi, d1i));
        v[t] = v0.x + v0.y;
        v[C + t] = v1.x + v1.y;
        if constexpr (kBlock) {
          const float2 sq = fma2(xr, xr, mul2(xi, xi));
          vs[t] = sq.x + sq.y;
        }
      }
      {
        constexpr int kShift = 5 - log2i<2 * C>();
        const float total = transpose_reduce<2 * C>(v, lane);
        if ((lane & ((1 << kShift) - 1)) == 0) S.warp_part[warp][lane >> kShift] = total;
      }
      if constexpr (kBlock) {
        constexpr int kShift = 5 - log2i<C>();
        const float total = transpose_reduce<C>(vs, lane);
        if ((lane & ((1 << kShift) - 1)) == 0) S.warp_part[warp][2 * C + (lane >> kShift)] = total;
      }
      // the CTA's sums, then (G > 1) every cluster CTA pushes them into every CTA's part_all
      // with asynchronous stores completing on the receiver's `red` barrier (no cluster barrier
      // in the loop; a barrier is re-armed for tile n + 2 once tile n's sums have arrived, and no
      // peer can push tile n + 2 before this CTA has pushed tile n + 1)
      __syncthreads();
      if (tid < kVals) {
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) sum += S.warp_part[w][tid];
        if (G > 1) {
          for (int rr = 0; rr < G; ++rr)
            st_async_f32(cluster_smem_addr(&S.part_all[buf][g][tid], (unsigned)rr), sum,
                         cluster_smem_addr(&S.red[buf], (unsigned)rr));
        } else {
          S.part_all[buf][0][tid] = sum;
        }
      }
      if (G > 1) {
        if (!mbar_wait_cluster(&S.red[buf], (unsigned)((n >> 1) & 1), p.max_spin << 4)) timed_out = true;
        if (tid == 0 && i + 2 * nk < p.tiles) mbar_arrive_expect_tx(&S.red[buf], red_bytes);
      } else {
        __syncthreads();
      }
      if (tid < C) {
        // the cluster CTAs' partials in rank order (the same sums in every CTA)
        float q0[8], q1[8], qs[8];
#pragma unroll
        for (int rr = 0; rr < 8; ++rr) {
          if (rr < G) {
            q0[rr] = S.part_all[buf][rr][tid];
            q1[rr] = S.part_all[buf][rr][C + tid];
            qs[rr] = kBlock ? S.part_all[buf][rr][2 * C + tid] : 0.0f;
          } else {
            q0[rr] = q1[rr] = qs[rr] = 0.0f;
          }
        }
        float ss = 0.0f;
#pragma unroll
        for (int rr = 0; rr < 8; ++rr) {
          p0 += q0[rr];
          p1 += q1[rr];
          ss += qs[rr];
        }
        // RMSNorm scale of the token (block): r = (mean x^2 + eps)^(-1/2)
        if constexpr (kBlock) rs = rsqrtf(fmaf(ss, 1.0f / (float)W, p.norm_eps));
      }
    }
    {
      if (tid < C) {
        // controls: eta = ln16 tanh(p1), delta = pi/2 tanh(p0); the scan-level mode takes
        // (p0, p1) = (delta, eta) as given (no gate: tau = 0)
        const float tau0 = kScan ? 0.0f : tanh_accurate(fmaf(rs, p0, bias0));
        const float tau1 = kScan ? 0.0f : tanh_accurate(fmaf(rs, p1, bias1));
        const float E = kScan ? expf(p1) : expf(kLn16 * tau1), delta = kScan ? p0 : kHalfPi * tau0;
        const float keep = (p.reset != nullptr && tid < r.nvalid && p.reset[r.b * T + r.t0 + tid]) ? 0.0f : 1.0f;
        TokenCtl tc;
        tc.ed = make_float4(E, E, delta, delta);
        tc.tau = make_float4(tau0, tau0, tau1, tau1);
        tc.keep = make_float4(keep, keep, rs, rs);
        tc.proj = make_float4(p0, p1, 0.0f, 0.0f);
        S.ctl[tid] = tc;
        if (g == 0 && tid < r.nvalid) p.ctl[r.b * T + r.t0 + tid] = tc;
      }
      __syncthreads();
    }

    // the chunk's aggregate map per mode (both of the thread's modes in packed lanes)
    auto body = [&](auto full_tag) {
      constexpr bool kFull = decltype(full_tag)::value;
      constexpr int kU = kFull ? token_unroll<C>() : 1;  // partial unrolling keeps the kernel's code in the i-cache
      Cx2 P = cx2(bcast2(1.0f), bcast2(0.0f)), Q = cx2(bcast2(0.0f), bcast2(0.0f));
#pragma unroll kU
      for (int t = 0; t < C; ++t) {
        if (kFull || t < r.nvalid) {
          float2 xr = Pair<TIO>::load(&xt[t][0][2 * tid]);
          float2 xi = Pair<TIO>::load(&xt[t][1][2 * tid]);
          if constexpr (kBlock) {  // the mixer's input is the normalised token x r w
            const float2 rr = make_float2(S.ctl[t].keep.z, S.ctl[t].keep.w);
            xr = mul2(xr, mul2(rr, mc.wre));
            xi = mul2(xi, mul2(rr, mc.wim));
          }
          const TokenCoef2 k = token_coef2<kFast, fwd_rot<kFast>(), kScan>(mc, S.ctl[t]);
          Q = cfma2(k.a, Q, cx2(mul2(k.gain, content2<kFast, kMode>(xr, lin)), mul2(k.gain, content2<kFast, kMode>(xi, lin))));
          P = cmul2(k.a, P);
        }
      }
      float4* ap = p.agg + (r.b * p.chunks + r.c) * (long long)p.Mp + m0;
      if (act0) __stcg(ap, make_float4(P.re.x, P.im.x, Q.re.x, Q.im.x));
      if (act1) __stcg(ap + 1, make_float4(P.re.y, P.im.y, Q.re.y, Q.im.y));
    };
    if (r.nvalid == C) body(std::true_type{});
    else body(std::false_type{});
    __syncthreads();  // the buffer and the shared arrays are free for the tile after next
  }
  if (timed_out) atomicOr(&p.ls->status, kStatusTimeout);
  cluster_sync_relaxed();  // no CTA leaves while a peer may still read its shared memory
}

// ------------------------------------------------------------------------------ replay
template <typename TIO, int C, bool kFast, bool kVec, int kMode>
__global__ void __launch_bounds__(kFwdThreads) mixer_fwd_replay_kernel(const __grid_constant__ FwdParams p) {
  constexpr bool kBlock = kMode == kModeBlock, kProj = proj_like<kMode>(), kScan = kMode == kModeScan;
  const bool lin = kProj && p.content_linear != 0;
  const int g = blockIdx.x;
  const int tid = threadIdx.x;
  const int M = p.M, W = p.W;
  const int mbase = g * kFwdModes;
  const int m0 = mbase + 2 * tid;
  const bool act0 = m0 < M, act1 = m0 + 1 < M;
  const long long B = p.B, T = p.T;
  const long long k0 = blockIdx.y, nk = gridDim.y;

  extern __shared__ __align__(128) unsigned char smem_raw[];
  RepSmem<TIO, C>& S = *reinterpret_cast<RepSmem<TIO, C>*>(smem_raw);

  ModeConst2 mc = pair_modes(load_mode(p.pp, m0, M, act0), load_mode(p.pp, m0 + 1, M, act1));
  if constexpr (kBlock) load_norm_weight(mc, p.norm_w, m0, M, act0, act1);
  const int lane = tid & 31, warp = tid >> 5;

  if (tid == 0) {
    mbar_init(&S.bar[0], 1);
    mbar_init(&S.bar[1], 1);
    mbar_init_fence();
  }
  __syncthreads();

  // Tile inputs in shared memory: x rows and the C token controls (thread 0's copies). The first
  // tile's go out before the wait: x and the controls come from kernels before the carry scan,
  // which have completed when this kernel starts (see pdl_wait).
  auto issue_tma = [&](long long i, int buf) {  // (thread 0)
    const TileRef r = tile_ref(i, B, T, C);
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&S.bar[buf], act_box_bytes<TIO, C, kFwdModes>() + (unsigned)sizeof(TokenCtl) * (unsigned)r.nvalid);
    tma_load_3d(&S.x[buf][0][0][0], &p.map_x, mbase, 0, (int)(r.b * T + r.t0), &S.bar[buf]);
    bulk_copy_g2s(&S.ctl[buf][0], p.ctl + r.b * T + r.t0, (unsigned)sizeof(TokenCtl) * (unsigned)r.nvalid, &S.bar[buf]);
  };
  if (p.use_tma && tid == 0 && k0 < p.tiles) issue_tma(k0, 0);

  pdl_wait();  // the carries (scan) are complete from here on

  auto issue = [&](long long i, int buf) {
    const TileRef r = tile_ref(i, B, T, C);
    const TIO* src = static_cast<const TIO*>(p.x) + (r.b * T + r.t0) * W;
    const TokenCtl* csrc = p.ctl + r.b * T + r.t0;
    if (p.use_tma) {
      if (tid == 0) issue_tma(i, buf);
    } else {
      load_act_rows<TIO, kFwdModes>(src, W, M, mbase, r.nvalid, S.x[buf], kFwdThreads);
      for (int t = tid; t < r.nvalid; t += kFwdThreads) S.ctl[buf][t] = csrc[t];
    }
  };
  if (k0 < p.tiles && !p.use_tma) issue(k0, 0);
  // the state carried into tile i at the thread's two modes: the scan's state at the end of the
  // previous chunk (h0 or zero at chunk 0), loaded straight into registers a tile ahead
  const bool carry16 = (reinterpret_cast<uintptr_t>(p.carry) & 15u) == 0;
  auto tile_hin = [&](long long i) -> Cx2 {
    const TileRef r = tile_ref(i, B, T, C);
    float2 h0 = make_float2(0.0f, 0.0f), h1 = h0;
    if (r.c > 0) {
      const float2* hs = p.carry + (r.b * p.chunks + (r.c - 1)) * (long long)M + m0;
      if (kVec && act1 && carry16) {  // (M even: the pair starts on a 16-byte boundary)
        const float4 v = __ldcg(reinterpret_cast<const float4*>(hs));
        h0 = make_float2(v.x, v.y);
        h1 = make_float2(v.z, v.w);
      } else {
        if (act0) h0 = __ldcg(hs);
        if (act1) h1 = __ldcg(hs + 1);
      }
    } else if (p.h0_r != nullptr) {
      if (act0) h0 = make_float2(p.h0_r[r.b * M + m0], p.h0_i[r.b * M + m0]);
      if (act1) h1 = make_float2(p.h0_r[r.b * M + m0 + 1], p.h0_i[r.b * M + m0 + 1]);
    }
    return cx2(make_float2(h0.x, h1.x), make_float2(h0.y, h1.y));
  };
  Cx2 hin_next = k0 < p.tiles ? tile_hin(k0) : cx2(bcast2(0.0f), bcast2(0.0f));
  bool timed_out = false;

  for (long long n = 0;; ++n) {
    const long long i = k0 + n * nk;
    if (i >= p.tiles) break;
    const int buf = (int)(n & 1);
    if (i + nk < p.tiles) issue(i + nk, buf ^ 1);
    Cx2 h = hin_next;
    if (i + nk < p.tiles) hin_next = tile_hin(i + nk);  // (in flight under this tile)
    const TileRef r = tile_ref(i, B, T, C);
    if (p.use_tma) {
      if (!mbar_wait(&S.bar[buf], (unsigned)((n >> 1) & 1), p.max_spin << 4)) timed_out = true;
    } else {
      __syncthreads();
    }
    const TIO(*xt)[2][kFwdModes] = S.x[buf];
    const TokenCtl* ctl = S.ctl[buf];
    TIO* yrow = static_cast<TIO*>(p.y) + (r.b * T + r.t0) * W;
    auto body = [&](auto full_tag) {
      constexpr bool kFull = decltype(full_tag)::value;
      constexpr int kU = kFull ? token_unroll<C>() : 1;
#pragma unroll kU
      for (int t = 0; t < C; ++t) {
        if (kFull || t < r.nvalid) {
          const float2 xr = Pair<TIO>::load(&xt[t][0][2 * tid]);
          const float2 xi = Pair<TIO>::load(&xt[t][1][2 * tid]);
          const TokenCoef2 k = token_coef2<kFast, fwd_rot<kFast>(), kScan>(mc, ctl[t]);
          if constexpr (kBlock) {
            // mixer input x r w; block output x + relu(h); relu bits for the backward
            const float2 rr = make_float2(ctl[t].keep.z, ctl[t].keep.w);
            const float2 nr = mul2(xr, mul2(rr, mc.wre)), ni = mul2(xi, mul2(rr, mc.wim));
            h = cfma2(k.a, h, cx2(mul2(k.gain, tanh_t2<kFast>(nr)), mul2(k.gain, tanh_t2<kFast>(ni))));
            store_sum_pair<TIO, kVec>(yrow + (long long)t * W, M, m0, act0, act1, xr, xi, h);
            if (p.states != nullptr)
              store_y_pair<TIO, kVec, false>(static_cast<TIO*>(p.states) + (r.b * T + r.t0 + t) * W, M, m0, act0,
                                             act1, make_float2(h.re.x, h.im.x), make_float2(h.re.y, h.im.y));
            store_relu_bits(p.mask + (r.b * T + r.t0 + t) * (long long)p.mask_words + (mbase >> 6) * 4 + warp * 4,
                            h, lane);
          } else {
            h = cfma2(k.a, h, cx2(mul2(k.gain, content2<kFast, kMode>(xr, lin)), mul2(k.gain, content2<kFast, kMode>(xi, lin))));
            if (kScan && p.y_im != nullptr) {
              // separate real and imaginary outputs, [B*T, M] each
              const long long o = (r.b * T + r.t0 + t) * (long long)M + m0;
              TIO* yr = static_cast<TIO*>(p.y) + o;
              TIO* yi = static_cast<TIO*>(p.y_im) + o;
              if (kVec && act1) {
                Pair<TIO>::store(yr, h.re.x, h.re.y);
                Pair<TIO>::store(yi, h.im.x, h.im.y);
              } else {
                if (act0) { Io<TIO>::store(yr, h.re.x); Io<TIO>::store(yi, h.im.x); }
                if (act1) { Io<TIO>::store(yr + 1, h.re.y); Io<TIO>::store(yi + 1, h.im.y); }
              }
            } else {
              store_y_pair<TIO, kVec, !kProj>(yrow + (long long)t * W, M, m0, act0, act1,
                                              make_float2(h.re.x, h.im.x), make_float2(h.re.y, h.im.y));
              if (!kProj && p.states != nullptr)
                store_y_pair<TIO, kVec, false>(static_cast<TIO*>(p.states) + (r.b * T + r.t0 + t) * W, M, m0, act0,
                                               act1, make_float2(h.re.x, h.im.x), make_float2(h.re.y, h.im.y));
            }
          }
        }
      }
    };
    if (r.nvalid == C) body(std::true_type{});
    else body(std::false_type{});
    __syncthreads();  // the buffer is free for the tile after next
  }
  if (timed_out) atomicOr(&p.ls->status, kStatusTimeout);
}
