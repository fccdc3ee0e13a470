// SPARC mixer forward / backward for B200 (sm_100a).
//
// Work unit ("tile"): one batch row b and one chunk of C consecutive tokens, all M modes; CTA g
// of a tile owns modes [g*256, g*256 + 256), two adjacent modes per thread. The forward is
//   summary  (cluster of G CTAs per tile) token controls + each chunk's affine map
//            h_out = P h_in + Q per mode,
//   scan     the chunk carries: a decoupled-lookback scan over segments of chunks,
//   replay   the recurrence inside every chunk from its carried-in state, y = relu(h);
// the backward mirrors it (reverse summary from the relu mask of y, reverse scan of the
// adjoint carries, gradient kernel) and ends with a fixed-order reduction of the per-cluster
// parameter-gradient partials. The tile kernels are persistent with a static schedule and
// never wait on each other; the only cross-CTA waits are the scan's bounded lookback polls.
// The forward's chunk carries and per-token controls are outputs the backward reads back.
//
// Parity targets (reference paths inside Botwwt/sparc):
//   controls  forward/control.py:129-139      write  forward/control.py:167-195
//   scan      forward/scan.py:886-1003,1277-1354  (chunk summary / prefix / replay)
//   backward  backward/scan.py:382-644 (reverse chunk kernels), backward/control.py:11-89
//             (write backward), autograd of make_controls for the controller gradient.
#include <cooperative_groups.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <type_traits>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "sparc_b200.h"
#include "timing.cuh"

namespace cg = cooperative_groups;

namespace sparc {

// Unrolling of the token loops of full chunks (0 = the whole chunk).
#ifndef SPARC_TOKEN_UNROLL
#define SPARC_TOKEN_UNROLL 4
#endif
template <int C>
__host__ __device__ constexpr int token_unroll() { return SPARC_TOKEN_UNROLL == 0 ? C : SPARC_TOKEN_UNROLL; }

// Tokens per chunk (the granularity of the saved carries): 16 for bfloat16, 8 for float32
// (whose shared-memory tiles are twice as large per token).
__host__ __device__ constexpr int chunk_for(int dtype) { return dtype == SPARC_DTYPE_BF16 ? 16 : 8; }

// What the tile kernels compute (their kMode template argument):
constexpr int kModePlain = 0;  // y = relu(SPARC(x)), controls projected from x (the torch module)
constexpr int kModeBlock = 1;  // y = x + relu(SPARC(RMSNorm(x))) (a pre-norm residual block)
constexpr int kModeProj = 2;   // h = SPARC states from a content input u [B, T, 2M] and given
                               // per-token controller projections p [B, T, 2] (the projection
                               // variant: u = x Wc and p = [x, 1] c come from matrix products)
constexpr int kModeScan = 3;   // h = SPARC states from given per-token controls (delta, eta)
                               // [B, T, 2] and writes b [B, T, 2M] (the reference's scan-level
                               // functions, sparc_scan and its kin): unit write gain, any eta and
                               // delta (the rotation is range-reduced)
// Modes whose output is the states themselves (no relu) from given per-token controls.
template <int kMode>
__host__ __device__ constexpr bool proj_like() { return kMode == kModeProj || kMode == kModeScan; }

// Content of a token: tanh(u), or u itself for a projection-mode layer with a linear content
// activation (lin, uniform over the launch).
template <bool kFast, int kMode>
__device__ __forceinline__ float2 content2(float2 u, bool lin) {
  if constexpr (kMode == kModeScan) {
    return u;  // the write itself
  } else {
    if constexpr (kMode == kModeProj) {
      if (lin) return u;
    }
    return tanh_t2<kFast>(u);
  }
}

// sin / cos of any float x by Cody and Waite's argument reduction: k = rint(x 2/pi),
// r = x - k pi/2 with pi/2 split into three parts (c1, c2 exact in 12 bits, so k c1 and k c2 are
// exact for |k| < 2^12; c3 the rest), |r| <= pi/4, then the series on [-pi/2, pi/2] and the
// quadrant k mod 4. (The scan-level mode's phase offset (1 - rho) delta is unbounded.)
__device__ __forceinline__ void sincos_reduced(float x, float* s, float* c) {
  const float k = rintf(x * 0.636619772f);
  float r = fmaf(-k, 1.5703125f, x);
  r = fmaf(-k, 4.8375129699707031e-4f, r);
  r = fmaf(-k, 7.5497901264043321e-8f, r);
  float sr, cr;
  sincos_halfpi(r, &sr, &cr);
  const int q = ((int)k) & 3;
  *s = q == 0 ? sr : q == 1 ? cr : q == 2 ? -sr : -cr;
  *c = q == 0 ? cr : q == 1 ? -sr : q == 2 ? -cr : sr;
}

struct ModeConst {
  float nu;      // e^{nu_log}
  float nl2e;    // nu * log2(e)
  float ct, st;  // cos/sin theta
  float theta;
  float gconst;  // e^{write_log_gain} / sqrt(-expm1(-2 nu))
  float stat;    // nu e^{-2nu} / -expm1(-2nu)
  float wpr, wrr;
  float d0r, d0i, d1r, d1i;  // controller directions at columns m and M+m
};

struct MixerParamPtrs {
  const float* nu_log;
  const float* theta_log;
  const float* phase_dir;   // [W+1]
  const float* radial_dir;  // [W+1]
  const float* wlg;
  const float* wpr;
  const float* wrr;
};

__device__ __forceinline__ ModeConst load_mode(const MixerParamPtrs& pp, int m, int M, bool active) {
  ModeConst mc;
  const float nu_log = active ? pp.nu_log[m] : 0.0f;
  const float theta_log = active ? pp.theta_log[m] : 0.0f;
  mc.nu = expf(nu_log);
  mc.nl2e = mc.nu * kLog2e;
  mc.theta = expf(theta_log);
  sincosf(mc.theta, &mc.st, &mc.ct);
  const float den = -expm1f(-2.0f * mc.nu);
  mc.gconst = active ? expf(pp.wlg[m]) * rsqrtf(den) : 0.0f;
  mc.stat = mc.nu * expf(-2.0f * mc.nu) / den;
  mc.wpr = active ? pp.wpr[m] : 0.0f;
  mc.wrr = active ? pp.wrr[m] : 0.0f;
  // (a projection-mode launch has no controller directions: its controls come precomputed)
  const bool dirs = active && pp.phase_dir != nullptr;
  mc.d0r = dirs ? pp.phase_dir[m] : 0.0f;
  mc.d0i = dirs ? pp.phase_dir[M + m] : 0.0f;
  mc.d1r = dirs ? pp.radial_dir[m] : 0.0f;
  mc.d1i = dirs ? pp.radial_dir[M + m] : 0.0f;
  return mc;
}

// Rotation e^{i phi}, phi = theta + (1 - rho) delta, by kRot: 0 the series of the bounded offset
// (1 - rho) delta (|.| <= pi/2) applied to the mode's e^{i theta}; 1 the hardware sin / cos of
// the whole angle; 2 the hardware sin / cos of the offset (inside their accurate range) applied
// to e^{i theta}.
template <int kRot, bool kScan = false>
__device__ __forceinline__ float2 transition_rot(const ModeConst& mc, float rho, float delta) {
  float s, c;
  if constexpr (kScan) {  // any delta: the reduced offset applied to e^{i theta}
    sincos_reduced(fmaf(-rho, delta, delta), &s, &c);
    const float rct = rho * mc.ct, rst = rho * mc.st;
    return make_float2(fmaf(rct, c, -rst * s), fmaf(rst, c, rct * s));
  } else if constexpr (kRot == 1) {
    sincos_hw(fmaf(-rho, delta, delta) + mc.theta, &s, &c);
    return make_float2(rho * c, rho * s);
  } else {
    if constexpr (kRot == 2) sincos_hw(fmaf(-rho, delta, delta), &s, &c);
    else sincos_halfpi(fmaf(-rho, delta, delta), &s, &c);
    const float rct = rho * mc.ct, rst = rho * mc.st;
    return make_float2(fmaf(rct, c, -rst * s), fmaf(rst, c, rct * s));
  }
}

// The per-(token, mode) coefficients, two modes at once (the lanes are the thread's modes m and
// m+1), with the float operations packed into f32x2 instructions; the hardware approximations
// stay per lane. The token's controls come as pairs (E, E), (delta, delta), (tau0, tau0),
// (tau1, tau1). kFast (bfloat16 activations): -expm1 from a shorter series and the gate from
// the hardware tanh (2 sigma(q) = 1 + tanh(q / 2)); otherwise (float32) every factor is accurate
// to a few ulp. The rotation follows kRot (transition_rot).
struct ModeConst2 {
  float2 nu, nl2e_neg, theta, ct, st, gconst, stat, wpr, wrr;
  float2 wpr_h, wrr_l;  // wpr * 2/pi, wrr / ln 16 (the gate's chain factors in the backward)
  float2 d0r, d0i, d1r, d1i;
  float2 wre, wim;      // RMSNorm weight at the modes' real / imaginary columns (1 outside a block)
};
__device__ __forceinline__ ModeConst2 pair_modes(const ModeConst& a, const ModeConst& b) {
  ModeConst2 m;
  m.nu = make_float2(a.nu, b.nu);
  m.nl2e_neg = make_float2(-a.nl2e, -b.nl2e);
  m.theta = make_float2(a.theta, b.theta);
  m.ct = make_float2(a.ct, b.ct);
  m.st = make_float2(a.st, b.st);
  m.gconst = make_float2(a.gconst, b.gconst);
  m.stat = make_float2(a.stat, b.stat);
  m.wpr = make_float2(a.wpr, b.wpr);
  m.wrr = make_float2(a.wrr, b.wrr);
  m.wpr_h = make_float2(a.wpr * kInvHalfPi, b.wpr * kInvHalfPi);
  m.wrr_l = make_float2(a.wrr * kInvLn16, b.wrr * kInvLn16);
  m.d0r = make_float2(a.d0r, b.d0r);
  m.d0i = make_float2(a.d0i, b.d0i);
  m.d1r = make_float2(a.d1r, b.d1r);
  m.d1i = make_float2(a.d1i, b.d1i);
  m.wre = m.wim = make_float2(1.0f, 1.0f);
  return m;
}

// The RMSNorm weight of a block at the thread's modes (columns m, m+1 and M+m, M+m+1).
__device__ __forceinline__ void load_norm_weight(ModeConst2& mc, const float* w, int m0, int M, bool a0, bool a1) {
  mc.wre = make_float2(a0 ? w[m0] : 0.0f, a1 ? w[m0 + 1] : 0.0f);
  mc.wim = make_float2(a0 ? w[M + m0] : 0.0f, a1 ? w[M + m0 + 1] : 0.0f);
}

// Per-token controls as the forward saves them (64 bytes): every value twice, so that a
// thread's two modes load them as packed pairs; keep is 0 at a token where a segment reset cuts
// the recurrence (its transition is zero), else 1.
struct TokenCtl {
  float4 ed;    // E, E, delta, delta   (E = e^eta)
  float4 tau;   // tau0, tau0, tau1, tau1
  float4 keep;  // keep, keep, r, r     (r: the token's RMSNorm scale in a block, else 1)
  float4 proj;  // q0, q1, 0, 0         (the projections before the scale r: the norm's backward)
};
static_assert(sizeof(TokenCtl) == 64, "token controls are four 16-byte words");

struct TokenCoef2 {
  float2 z, rho;
  Cx2 a;
  float2 num, gate, gain;
};

// kRot (see transition_rot): 1 the hardware sin / cos of the whole angle (MUFU pipe), 0 the
// series of the bounded offset (FMA pipe), 2 the hardware sin / cos of the offset; by default
// the fast path's choice (1 for bfloat16, 0 for float32).
// The transition a = rk e^{i(theta + (1 - rho) delta)} of two modes (rk = rho keep: 0 at a
// reset), the rotation by kRot; the scan-level mode (kScan) takes any delta (reduced offset).
template <int kRot, bool kScan>
__device__ __forceinline__ Cx2 transition2(const ModeConst2& mc, float2 rho, float2 rk, float2 delta) {
  if constexpr (kScan) {
    const float2 off = sub2(delta, mul2(rho, delta));
    float2 sn, cs;
    sincos_reduced(off.x, &sn.x, &cs.x);
    sincos_reduced(off.y, &sn.y, &cs.y);
    const float2 rct = mul2(rk, mc.ct), rst = mul2(rk, mc.st);
    return Cx2{sub2(mul2(rct, cs), mul2(rst, sn)), fma2(rst, cs, mul2(rct, sn))};
  } else if constexpr (kRot == 1) {
    const float2 ph = sub2(add2(delta, mc.theta), mul2(rho, delta));  // theta + (1 - rho) delta
    float2 sn, cs;
    sincos_hw(ph.x, &sn.x, &cs.x);
    sincos_hw(ph.y, &sn.y, &cs.y);
    return Cx2{mul2(rk, cs), mul2(rk, sn)};
  } else {
    float2 sn, cs;
    const float2 off = sub2(delta, mul2(rho, delta));  // (1 - rho) delta, |.| <= pi/2
    if constexpr (kRot == 2) {
      sincos_hw(off.x, &sn.x, &cs.x);
      sincos_hw(off.y, &sn.y, &cs.y);
    } else {
      sincos_halfpi2(off, &sn, &cs);
    }
    const float2 rct = mul2(rk, mc.ct), rst = mul2(rk, mc.st);
    return Cx2{sub2(mul2(rct, cs), mul2(rst, sn)), fma2(rst, cs, mul2(rct, sn))};
  }
}

template <bool kFast, int kRot = kFast ? 1 : 0, bool kScan = false>
__device__ __forceinline__ TokenCoef2 token_coef2(const ModeConst2& mc, float2 E, float2 delta, float2 tau0,
                                                  float2 tau1, float2 keep) {
  TokenCoef2 k;
  k.z = mul2(mc.nu, E);
  k.rho = ex2_2(mul2(mc.nl2e_neg, E));
  k.a = transition2<kRot, kScan>(mc, k.rho, mul2(k.rho, keep), delta);
  if constexpr (kScan) {  // the write is b itself (unit gain)
    k.num = k.gate = k.gain = bcast2(1.0f);
    return k;
  }
  const float2 q = fma2(tau0, mc.wpr, mul2(tau1, mc.wrr));
  const float2 u = add2(k.z, k.z);
  if constexpr (kFast) {
    const float2 ser = mul2(u, fma2(fma2(fma2(bcast2(-4.1666666666666667e-2f), u, bcast2(1.6666666666666667e-1f)), u,
                                         bcast2(-0.5f)), u, bcast2(1.0f)));
    const float2 big = sub2(bcast2(1.0f), mul2(k.rho, k.rho));
    k.num = make_float2(u.x < 0.25f ? ser.x : big.x, u.y < 0.25f ? ser.y : big.y);
    k.gate = add2(bcast2(1.0f), tanh_hw2(mul2(bcast2(0.5f), q)));
  } else {
    k.num = one_minus_exp_neg2(u, mul2(k.rho, k.rho));
    const float2 r = rcp_2(add2(bcast2(1.0f), ex2_2(mul2(bcast2(-kLog2e), q))));
    k.gate = add2(r, r);
  }
  k.gain = mul2(mul2(mc.gconst, sqrt_2(k.num)), k.gate);
  return k;
}

// The same from a saved controls record.
template <bool kFast, int kRot = kFast ? 1 : 0, bool kScan = false>
__device__ __forceinline__ TokenCoef2 token_coef2(const ModeConst2& mc, const TokenCtl& c) {
  return token_coef2<kFast, kRot, kScan>(mc, make_float2(c.ed.x, c.ed.y), make_float2(c.ed.z, c.ed.w),
                                         make_float2(c.tau.x, c.tau.y), make_float2(c.tau.z, c.tau.w),
                                         make_float2(c.keep.x, c.keep.y));
}

// Transition a = rho e^{i(theta + (1-rho) delta)} alone (the reverse local pass needs no write).
template <bool kFast, int kRot = kFast ? 1 : 0, bool kScan = false>
__device__ __forceinline__ float2 token_transition(const ModeConst& mc, float E, float delta, float keep) {
  const float2 a = transition_rot<kRot, kScan>(mc, ex2_approx(-mc.nl2e * E), delta);
  return make_float2(a.x * keep, a.y * keep);
}

// Warp transpose-reduce of N values per lane (N a power of two, N <= 32). Afterwards lane l
// holds the warp total of value l >> (5 - log2 N).
template <int N>
__device__ __forceinline__ float transpose_reduce(float (&v)[N], int lane) {
  static_assert(N >= 1 && N <= 32 && (N & (N - 1)) == 0, "N must be a power of two <= 32");
  int n = N;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    if (n > 1) {
      const bool upper = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < N / 2; ++i) {
        if (i < n / 2) {
          const float send = upper ? v[i] : v[i + n / 2];
          const float keep = upper ? v[i + n / 2] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      n >>= 1;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    }
  }
  return v[0];
}

template <int N>
__host__ __device__ constexpr int log2i() { return N <= 1 ? 0 : 1 + log2i<N / 2>(); }

// ------------------------------------------------------------------------------ carry scan
// Per (row b, mode m): v_j = A_j v_{j-1} + B_j over the chunks j in processing order (forward:
// chunk j; backward: chunk chunks-1-j), v_{-1} = init (h0, or the gradient of the returned last
// state; else 0). out[chunk] receives every v; `final` (optional) the last one (the forward's
// last state, the backward's gradient of h0).
//
// One thread-block cluster of kScanQ CTAs of kScanWarps warps per (row, 32 modes): lane l owns
// mode m0 + l, and the cluster's kScanQ x kScanWarps warps own consecutive spans of
// L = ceil(chunks / spans) chunks (warp w of CTA q: span q kScanWarps + w). Each lane composes its
// span's maps (the first kScanHold of them kept in registers), leaves the span's map in shared
// memory, and after one cluster barrier composes the earlier spans' maps in order (its own CTA's
// from shared memory, the earlier CTAs' through distributed shared memory) into its carry-in;
// then it walks its span writing every chunk's v. A warp's 32 lanes read 32 consecutive maps
// (512 contiguous bytes) per chunk. The composition order is fixed, so the carries are bitwise
// reproducible; nothing waits but the cluster barriers.
// Rotation choice per kernel family and activation type (transition_rot): bfloat16 kernels use
// the hardware sin / cos of the whole angle; the float32 forward the series of the bounded
// offset (its outputs agree with the decode step's libm to ~1e-7); the float32 backward the
// hardware sin / cos of the offset (absolute error ~5e-7, inside [-pi/2, pi/2], far below the
// 1e-3 gradient tolerance; 4% faster gradient kernel). SPARC_F32_ROT_FWD / _BWD select 0 (series)
// or 2 (hardware offset); SPARC_FWD_HW_ROTATION 0 makes the bfloat16 forward use the series.
#ifndef SPARC_FWD_HW_ROTATION
#define SPARC_FWD_HW_ROTATION 1
#endif
#ifndef SPARC_F32_ROT_FWD
#define SPARC_F32_ROT_FWD 0
#endif
#ifndef SPARC_F32_ROT_BWD
#define SPARC_F32_ROT_BWD 2
#endif
template <bool kFast>
__host__ __device__ constexpr int fwd_rot() { return kFast ? (SPARC_FWD_HW_ROTATION ? 1 : 0) : SPARC_F32_ROT_FWD; }
template <bool kFast>
__host__ __device__ constexpr int bwd_rot() { return kFast ? 1 : SPARC_F32_ROT_BWD; }

#ifndef SPARC_SCAN_Q
#define SPARC_SCAN_Q 4
#endif
#ifndef SPARC_SCAN_WARPS
#define SPARC_SCAN_WARPS 4
#endif
constexpr int kScanQ = SPARC_SCAN_Q;            // CTAs per (row, 32 modes): a portable cluster
constexpr int kScanWarps = SPARC_SCAN_WARPS;    // spans per CTA
constexpr int kScanSpans = kScanQ * kScanWarps;
constexpr int kScanThreads = 32 * kScanWarps;
constexpr int kScanHold = 16;                   // span maps held in registers (longer spans reload)

struct ScanParams {
  const float4* agg;     // [B, chunks, Mp] per-chunk maps (A, B)
  float2* out;           // [B, chunks, M]
  const float* init_r;   // [B, M] or null
  const float* init_i;
  float* final_r;        // [B, M] or null
  float* final_i;
  int M, Mp, chunks, span;
  int reverse;
};

__global__ void __launch_bounds__(kScanThreads) mixer_carry_scan_kernel(const ScanParams p) {
  __shared__ float4 s_map[kScanWarps][32];  // this CTA's span maps per mode (peers read them)
  cg::cluster_group cluster = cg::this_cluster();
  const int q = (int)cluster.block_rank();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int sp = q * kScanWarps + w;  // this warp's span
  const long long b = blockIdx.y;
  const int m = (blockIdx.x / kScanQ) * 32 + lane;
  const bool act = m < p.M;
  const int j0 = min(sp * p.span, p.chunks), j1 = min(j0 + p.span, p.chunks);
  // chunk maps and outputs of processing index j: strided pointers from the span's first chunk
  const long long c0 = p.reverse ? p.chunks - 1 - j0 : j0;
  const long long step = p.reverse ? -1 : 1;
  const float4* ap = p.agg + (b * p.chunks + c0) * (long long)p.Mp + m;
  float2* op = p.out + (b * p.chunks + c0) * (long long)p.M + m;
  const long long astep = step * p.Mp, ostep = step * p.M;
  const float4 ident = make_float4(1.0f, 0.0f, 0.0f, 0.0f);
  pdl_wait();  // the chunk maps (summary) are complete from here on

  // the span's map; its first kScanHold maps stay in registers for the walk
  float4 held[kScanHold];
#pragma unroll
  for (int u = 0; u < kScanHold; ++u) held[u] = (act && j0 + u < j1) ? __ldcg(ap + u * astep) : ident;
  float2 A = make_float2(1.0f, 0.0f), Bv = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int u = 0; u < kScanHold; ++u) {
    Bv = cfma(make_float2(held[u].x, held[u].y), Bv, make_float2(held[u].z, held[u].w));
    A = cmul(make_float2(held[u].x, held[u].y), A);
  }
  for (int j = j0 + kScanHold; j < j1; j += kScanHold) {
    float4 a[kScanHold];
#pragma unroll
    for (int u = 0; u < kScanHold; ++u) a[u] = (act && j + u < j1) ? __ldcg(ap + (j - j0 + u) * astep) : ident;
#pragma unroll
    for (int u = 0; u < kScanHold; ++u) {
      Bv = cfma(make_float2(a[u].x, a[u].y), Bv, make_float2(a[u].z, a[u].w));
      A = cmul(make_float2(a[u].x, a[u].y), A);
    }
  }
  s_map[w][lane] = make_float4(A.x, A.y, Bv.x, Bv.y);
  cluster.sync();

  // carry into the span: init, then the earlier spans' maps in order
  float2 v = make_float2(0.0f, 0.0f);
  if (p.init_r != nullptr && act) v = make_float2(p.init_r[b * p.M + m], p.init_i[b * p.M + m]);
  {  // the earlier CTAs' spans: every read issued before the first composition
    float4 mk[kScanQ - 1][kScanWarps];
#pragma unroll
    for (int k = 0; k < kScanQ - 1; ++k) {
      if (k < q) {
        const float4* peer = cluster.map_shared_rank(&s_map[0][0], k);
#pragma unroll
        for (int u = 0; u < kScanWarps; ++u) mk[k][u] = peer[u * 32 + lane];
      }
    }
#pragma unroll
    for (int k = 0; k < kScanQ - 1; ++k) {
      if (k < q) {
#pragma unroll
        for (int u = 0; u < kScanWarps; ++u)
          v = cfma(make_float2(mk[k][u].x, mk[k][u].y), v, make_float2(mk[k][u].z, mk[k][u].w));
      }
    }
  }
  for (int u = 0; u < w; ++u) {  // this CTA's earlier spans
    const float4 mk = s_map[u][lane];
    v = cfma(make_float2(mk.x, mk.y), v, make_float2(mk.z, mk.w));
  }

  // walk the span
#pragma unroll
  for (int u = 0; u < kScanHold; ++u) {
    if (j0 + u < j1) {
      v = cfma(make_float2(held[u].x, held[u].y), v, make_float2(held[u].z, held[u].w));
      if (act) op[u * ostep] = v;
    }
  }
  for (int j = j0 + kScanHold; j < j1; j += kScanHold) {
    float4 a[kScanHold];
#pragma unroll
    for (int u = 0; u < kScanHold; ++u) a[u] = (act && j + u < j1) ? __ldcg(ap + (j - j0 + u) * astep) : ident;
#pragma unroll
    for (int u = 0; u < kScanHold; ++u) {
      if (j + u < j1) {
        v = cfma(make_float2(a[u].x, a[u].y), v, make_float2(a[u].z, a[u].w));
        if (act) op[(j - j0 + u) * ostep] = v;
      }
    }
  }
  if (p.final_r != nullptr && act && j0 < j1 && j1 == p.chunks) {
    p.final_r[b * p.M + m] = v.x;
    p.final_i[b * p.M + m] = v.y;
  }
  cluster_sync_relaxed();  // no CTA leaves while a peer may still read its span maps
}

#include "mixer_fwd.cuh"

#include "mixer_bwd.cuh"

struct ReduceParams {
  const double* part;
  int clusters, Mp, M, W;
  const float* theta_log;
  float* g_nu_log;
  float* g_theta_log;
  float* g_wlg;
  float* g_wpr;
  float* g_wrr;
  float* g_energy;
  float* g_phase_dir;   // [W+1], or null (projection mode)
  float* g_radial_dir;  // [W+1], or null (projection mode)
  float* g_norm_w;      // [W] (block) or null
  PeerExchange xchg;    // world > 1: sum every gradient over the ranks before writing it
};

// grid (ceil(Mp/32), kPartModes + 1), block (32, kReduceWarps). Rows q < kPartModes: warp w sums
// clusters w, w + kReduceWarps, ... for 32 modes (coalesced, eight loads in flight), then warp 0
// adds the warps' sums. Row kPartModes (block 0 only): warps 0 and 1 sum the two controller
// biases over the clusters, lane-strided, then a shuffle tree. Every order is fixed. With an
// exchange group (N GPUs of batch-sharded data parallelism), warp 0 of every CTA then sums its
// values over the ranks through NVLink peer memory (warp_exchange) before writing them: the
// gradient reduction and the cross-GPU all-reduce are one kernel.
constexpr int kReduceWarps = 16;
constexpr int kReduceUnroll = 8;

__global__ void __launch_bounds__(32 * kReduceWarps) mixer_reduce_kernel(const ReduceParams r) {
  pdl_wait();  // the partials (gradient kernel) are complete from here on
  const int lane = threadIdx.x, w = threadIdx.y;
  const int q = blockIdx.y;
  const bool xchg = r.xchg.world > 1;
  const int slot = blockIdx.y * gridDim.x + blockIdx.x;  // this CTA's exchange slot
  if (q == kPartModes) {
    // (uniform per CTA, and across the ranks, which all run the same configuration)
    if (blockIdx.x != 0 || r.g_phase_dir == nullptr) return;
    __shared__ float sb[2];
    if (w < 2) {
      const double* pb = r.part + (long long)r.clusters * kPartModes * r.Mp;
      double t = 0.0;
      for (int k = lane; k < r.clusters; k += 32) t += pb[2 * k + w];
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      if (lane == 0) sb[w] = (float)t;
    }
    __syncthreads();
    if (w == 0) {
      float v = lane < 2 ? sb[lane] : 0.0f;
      if (xchg) v = warp_exchange(r.xchg, slot, v);
      if (lane < 2) (lane == 0 ? r.g_phase_dir : r.g_radial_dir)[r.W] = v;
    }
    return;
  }
  // rows without a destination (directions in projection mode, norm weight outside a block)
  if ((q >= 5 && q <= 8 && r.g_phase_dir == nullptr) || (q >= 9 && r.g_norm_w == nullptr)) return;
  const int m = blockIdx.x * 32 + lane;
  __shared__ double sm[kReduceWarps][32];
  double s8[kReduceUnroll];
#pragma unroll
  for (int u = 0; u < kReduceUnroll; ++u) s8[u] = 0.0;
  if (m < r.Mp) {
    int k = w;
    for (; k + (kReduceUnroll - 1) * kReduceWarps < r.clusters; k += kReduceUnroll * kReduceWarps) {
#pragma unroll
      for (int u = 0; u < kReduceUnroll; ++u)
        s8[u] += r.part[((long long)(k + u * kReduceWarps) * kPartModes + q) * r.Mp + m];
    }
    for (; k < r.clusters; k += kReduceWarps) s8[0] += r.part[((long long)k * kPartModes + q) * r.Mp + m];
  }
  double sw = 0.0;
#pragma unroll
  for (int u = 0; u < kReduceUnroll; ++u) sw += s8[u];
  sm[w][lane] = sw;
  __syncthreads();
  if (w != 0) return;
  const bool ok = m < r.M;
  float v = 0.0f;
  if (ok) {
    double t = 0.0;
#pragma unroll
    for (int i = 0; i < kReduceWarps; ++i) t += sm[i][lane];
    v = q == 1 ? (float)(t * exp((double)r.theta_log[m])) : (float)t;
  }
  // N ranks: the whole warp exchanges its 32 values over peer memory; every rank gets the sum
  if (xchg) v = warp_exchange(r.xchg, slot, v);
  if (!ok) return;
  switch (q) {
    case 0: r.g_nu_log[m] = v; r.g_energy[m] = 0.0f; break;
    case 1: r.g_theta_log[m] = v; break;
    case 2: r.g_wlg[m] = v; break;
    case 3: r.g_wpr[m] = v; break;
    case 4: r.g_wrr[m] = v; break;
    case 5: r.g_phase_dir[m] = v; break;
    case 6: r.g_phase_dir[r.M + m] = v; break;
    case 7: r.g_radial_dir[m] = v; break;
    case 8: r.g_radial_dir[r.M + m] = v; break;
    case 9: r.g_norm_w[m] = v; break;
    default: r.g_norm_w[r.M + m] = v; break;
  }
}

// ------------------------------------------------------------------------------ host side
struct Plan {
  int dtype, C, chunks;
  int mode;                // kModePlain, kModeBlock, kModeProj or kModeScan
  long long tiles;         // B * chunks
  int G, Mp;               // CTAs of 256 modes per tile; modes padded to G * 256
  bool vec, tma;
  int sum_clusters, rep_rows, rsum_rows, grad_clusters, saved_clusters;
  size_t sum_smem, rep_smem, rsum_smem, grad_smem, saved_smem;
  long long scan_rows;     // carry-scan grid rows: B
  int scan_span;           // chunks per carry-scan span (warp)
};

static thread_local char g_err[512];
static void set_err(const char* msg) { snprintf(g_err, sizeof(g_err), "%s", msg); }

int fail(int code, const char* msg) {
  set_err(msg);
  return code;
}

static bool set_smem(const void* kernel, size_t dyn) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return true;
}

// Resident clusters of G CTAs (whole GPU) for a cluster kernel.
static int max_clusters(const void* kernel, int G, int NT, size_t dyn_smem) {
  if (G > 8) cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (!set_smem(kernel, dyn_smem)) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G, 1, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = dyn_smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = G;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

// Resident CTAs (whole GPU) for a plain kernel.
static int max_blocks(const void* kernel, int NT, size_t dyn_smem) {
  if (dyn_smem > 0 && !set_smem(kernel, dyn_smem)) return 0;
  int per_sm = 0, dev = 0, sms = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, NT, dyn_smem) != cudaSuccess ||
      cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return per_sm * sms;
}

// Kernel instances per activation type (bfloat16 uses the hardware tanh; float32 the accurate
// one) and mode (kModePlain, kModeBlock, kModeProj, kModeScan).
template <typename TIO>
struct Kernels {
  static constexpr bool kFast = std::is_same<TIO, __nv_bfloat16>::value;
  static constexpr int C = chunk_for(kFast ? SPARC_DTYPE_BF16 : SPARC_DTYPE_F32);
  template <int kM>
  static const void* sum_m() { return (const void*)mixer_fwd_summary_kernel<TIO, C, kFast, kM>; }
  template <int kM>
  static const void* rep_m(bool vec) {
    return vec ? (const void*)mixer_fwd_replay_kernel<TIO, C, kFast, true, kM>
               : (const void*)mixer_fwd_replay_kernel<TIO, C, kFast, false, kM>;
  }
  template <int kM>
  static const void* rsum_m() { return (const void*)mixer_bwd_summary_kernel<TIO, C, kFast, kM>; }
  template <int kM>
  static const void* grad_m(bool vec) {
    return vec ? (const void*)mixer_bwd_grad_kernel<TIO, C, kFast, true, kM>
               : (const void*)mixer_bwd_grad_kernel<TIO, C, kFast, false, kM>;
  }
  static const void* sum(int mode) {
    return mode == kModeBlock ? sum_m<kModeBlock>() : mode == kModeProj ? sum_m<kModeProj>()
         : mode == kModeScan ? sum_m<kModeScan>() : sum_m<kModePlain>();
  }
  static const void* rep(bool vec, int mode) {
    return mode == kModeBlock ? rep_m<kModeBlock>(vec) : mode == kModeProj ? rep_m<kModeProj>(vec)
         : mode == kModeScan ? rep_m<kModeScan>(vec) : rep_m<kModePlain>(vec);
  }
  static const void* rsum(int mode) {
    return mode == kModeBlock ? rsum_m<kModeBlock>() : mode == kModeProj ? rsum_m<kModeProj>()
         : mode == kModeScan ? rsum_m<kModeScan>() : rsum_m<kModePlain>();
  }
  static const void* grad(bool vec, int mode) {
    return mode == kModeBlock ? grad_m<kModeBlock>(vec) : mode == kModeProj ? grad_m<kModeProj>(vec)
         : mode == kModeScan ? grad_m<kModeScan>(vec) : grad_m<kModePlain>(vec);
  }
  template <int kM, int kSplit>
  static const void* saved_s(bool vec) {
    return vec ? (const void*)mixer_bwd_grad_saved_kernel<TIO, C, kSplit, kFast, true, kM>
               : (const void*)mixer_bwd_grad_saved_kernel<TIO, C, kSplit, kFast, false, kM>;
  }
  template <int kM>
  static const void* saved_m(bool vec, int G) { return G == 1 ? saved_s<kM, 2>(vec) : saved_s<kM, 1>(vec); }
  // halves for a CTA of its own (G == 1), whole tiles in clusters; (the scan-level mode has no
  // saved states: its outputs are two separate planes)
  static const void* saved(bool vec, int mode, int G) {
    return mode == kModeBlock ? saved_m<kModeBlock>(vec, G) : mode == kModeProj ? saved_m<kModeProj>(vec, G)
         : mode == kModeScan ? nullptr : saved_m<kModePlain>(vec, G);
  }
  static int saved_split(int G) { return G == 1 ? 2 : 1; }
  static size_t sum_smem() { return sizeof(SumSmem<TIO, C>); }
  static size_t rep_smem() { return sizeof(RepSmem<TIO, C>); }
  static size_t rsum_smem(int mode) {
    return mode == kModePlain ? sizeof(RsumSmem<TIO, C, true>) : sizeof(RsumSmem<TIO, C, false>);
  }
  static size_t grad_smem() { return sizeof(GradSmem<TIO, C>); }
  static size_t saved_smem(int G) { return G == 1 ? sizeof(GradSavedSmem<TIO, C, 2>) : sizeof(GradSavedSmem<TIO, C, 1>); }
};

template <typename TIO>
static void plan_kernels(Plan* pl, const void** k) {
  using K = Kernels<TIO>;
  pl->sum_smem = K::sum_smem();
  pl->rep_smem = K::rep_smem();
  pl->rsum_smem = K::rsum_smem(pl->mode);
  pl->grad_smem = K::grad_smem();
  pl->saved_smem = K::saved_smem(pl->G);
  k[0] = K::sum(pl->mode);
  k[1] = K::rep(pl->vec, pl->mode);
  k[2] = K::rsum(pl->mode);
  k[3] = K::grad(pl->vec, pl->mode);
  k[4] = K::saved(pl->vec, pl->mode, pl->G);
}

static int make_plan(long long B, long long T, int W, int dtype, int mode, Plan* pl) {
  if (B <= 0 || T <= 0 || W <= 0) { set_err("batch, length and width must be positive"); return SPARC_ERR_SHAPE; }
  if (W % 2) { set_err("SPARC rnn_width must be even"); return SPARC_ERR_SHAPE; }
  if (dtype != SPARC_DTYPE_F32 && dtype != SPARC_DTYPE_BF16) { set_err("unsupported dtype"); return SPARC_ERR_DTYPE; }
  const int M = W / 2;
  if (M > 8 * kFwdModes) { set_err("width above 4096 is not supported"); return SPARC_ERR_SHAPE; }
  pl->dtype = dtype;
  pl->mode = mode;
  pl->C = chunk_for(dtype);
  pl->chunks = (int)((T + pl->C - 1) / pl->C);
  pl->tiles = B * pl->chunks;
  if (pl->tiles >= (1LL << 31)) { set_err("too many tiles"); return SPARC_ERR_SHAPE; }
  pl->G = (M + kFwdModes - 1) / kFwdModes;
  pl->Mp = pl->G * kFwdModes;
  pl->vec = (M % 2) == 0;
  const size_t s = dtype == SPARC_DTYPE_BF16 ? 2 : 4;
  pl->tma = ((size_t)W * s) % 16 == 0 && ((size_t)M * s) % 16 == 0 && B * T < (1LL << 31);
  pl->scan_rows = B;
  pl->scan_span = (pl->chunks + kScanSpans - 1) / kScanSpans;
  if (pl->scan_rows > 65535) { set_err("batch too large for the carry scan's grid"); return SPARC_ERR_SHAPE; }

  const void* k[5];
  if (dtype == SPARC_DTYPE_BF16) plan_kernels<__nv_bfloat16>(pl, k);
  else plan_kernels<float>(pl, k);

  int dev = 0;
  cudaGetDevice(&dev);
  struct Key { int dev, dtype, G, vec, mode; int sum, rep, rsum, grad, saved; };
  static std::mutex mu;
  static Key cache[64];
  static int ncache = 0;
  std::lock_guard<std::mutex> lock(mu);
  const Key* hit = nullptr;
  for (int i = 0; i < ncache; ++i) {
    const Key& kk = cache[i];
    if (kk.dev == dev && kk.dtype == dtype && kk.G == pl->G && kk.vec == (int)pl->vec && kk.mode == mode) hit = &kk;
  }
  Key key;
  if (hit != nullptr) {
    key = *hit;
  } else {
    key = Key{dev, dtype, pl->G, (int)pl->vec, mode, 0, 0, 0, 0, 0};
    key.sum = max_clusters(k[0], pl->G, kFwdThreads, pl->sum_smem);
    key.rep = max_blocks(k[1], kFwdThreads, pl->rep_smem);
    key.rsum = max_blocks(k[2], kBwdThreads, pl->rsum_smem);
    key.grad = max_clusters(k[3], pl->G, kGradThreads, pl->grad_smem);
    key.saved = k[4] != nullptr ? max_clusters(k[4], pl->G, kGradThreads, pl->saved_smem) : 1;
    if (key.sum <= 0 || key.rep <= 0 || key.rsum <= 0 || key.grad <= 0 || key.saved <= 0) {
      set_err("occupancy query failed");
      return SPARC_ERR_LAUNCH;
    }
    if (ncache < 64) cache[ncache++] = key;
  }
  auto clamp = [](long long n, long long hi) { return (int)std::max<long long>(1, std::min<long long>(n, hi)); };
  pl->sum_clusters = clamp(key.sum, pl->tiles);
  pl->rep_rows = clamp(key.rep / pl->G, pl->tiles);
  pl->rsum_rows = clamp(key.rsum / pl->G, pl->tiles);
  pl->grad_clusters = clamp(key.grad, pl->tiles);
  pl->saved_clusters = clamp(key.saved, pl->tiles);
  return SPARC_OK;
}

struct WsLayout {
  size_t agg, kout, part, total;
};

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

static WsLayout ws_layout(const Plan& pl, long long B, int M) {
  WsLayout L;
  size_t off = align256(sizeof(LaunchState));
  L.agg = off;
  off = align256(off + (size_t)pl.tiles * pl.Mp * sizeof(float4));
  L.kout = off;
  off = align256(off + (size_t)B * pl.chunks * M * sizeof(float2));
  L.part = off;
  const size_t clusters = (size_t)std::max(pl.grad_clusters, pl.saved_clusters);  // (either gradient kernel)
  off = align256(off + (clusters * kPartModes * pl.Mp + 2 * clusters) * sizeof(double));
  L.total = off;
  return L;
}

// Every mixer launch carries a programmatic-stream-serialisation attribute: it may be scheduled
// while the previous kernel on the stream drains, and waits (pdl_wait) before reading that
// kernel's outputs.
template <typename P>
static cudaError_t launch_ex(const void* kernel, dim3 grid, dim3 block, int cluster_x, size_t dyn, cudaStream_t s,
                             const P& params) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = dyn;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = 1;
  ++na;
  if (cluster_x > 0) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = cluster_x;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  void* args[] = {const_cast<P*>(&params)};
  return cudaLaunchKernelExC(&cfg, kernel, args);
}

template <typename P>
static cudaError_t launch_cluster(const void* kernel, int G, int NT, int clusters, size_t dyn, cudaStream_t s,
                                  const P& params) {
  return launch_ex(kernel, dim3(G, clusters, 1), dim3(NT, 1, 1), G, dyn, s, params);
}

template <typename P>
static cudaError_t launch_plain(const void* kernel, dim3 grid, int NT, size_t dyn, cudaStream_t s, const P& params) {
  return launch_ex(kernel, grid, dim3(NT, 1, 1), 0, dyn, s, params);
}

static bool aligned16(const void* p) { return p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 == 0; }

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

// Activations [rows, W] seen as [rows][re|im half][M]: dims {M, 2, rows}, byte strides
// {M*s, W*s}; one box {256 modes, 2 halves, C rows} is a tile's shared-memory [C][2][256] array.
static bool act_tensor_map(CUtensorMap* map, const void* base, int dtype, long long rows, int M, int W, int C) {
  const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (enc == nullptr || base == nullptr) return false;
  const cuuint64_t s = dtype == SPARC_DTYPE_BF16 ? 2 : 4;
  const cuuint64_t dims[3] = {(cuuint64_t)M, 2, (cuuint64_t)rows};
  const cuuint64_t strides[2] = {(cuuint64_t)M * s, (cuuint64_t)W * s};
  const cuuint32_t box[3] = {(cuuint32_t)kFwdModes, 2, (cuuint32_t)C};
  const cuuint32_t estride[3] = {1, 1, 1};
  const CUresult r = enc(map, dtype == SPARC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                         3, const_cast<void*>(base), dims, strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static ScanParams scan_params(const Plan& pl, const WsLayout& L, char* ws, int M, int reverse,
                              const float* init_r, const float* init_i, float* final_r, float* final_i,
                              float2* out) {
  ScanParams sp;
  sp.agg = reinterpret_cast<const float4*>(ws + L.agg);
  sp.out = out;
  sp.init_r = init_r;
  sp.init_i = init_i;
  sp.final_r = final_r;
  sp.final_i = final_i;

  sp.M = M;
  sp.Mp = pl.Mp;
  sp.chunks = pl.chunks;
  sp.span = pl.scan_span;
  sp.reverse = reverse;
  return sp;
}

static cudaError_t launch_scan(const Plan& pl, const ScanParams& sp, cudaStream_t s) {
  // grid: kScanQ CTAs per 32 modes (x), rows (y); one cluster per (row, 32 modes)
  return launch_ex((const void*)mixer_carry_scan_kernel, dim3(kScanQ * ((sp.M + 31) / 32), (unsigned)pl.scan_rows),
                   dim3(kScanThreads, 1, 1), kScanQ, 0, s, sp);
}

// The carry scan for other users of chunk maps (the generic complex scan): maps [rows, chunks,
// M] float4, no initial state, spans as the mixer plans them.
cudaError_t launch_chunk_carry_scan(const float4* maps, float2* out, int rows, int M, int chunks, int reverse,
                                    float* final_r, float* final_i, cudaStream_t s) {
  ScanParams sp;
  sp.agg = maps;
  sp.out = out;
  sp.init_r = nullptr;
  sp.init_i = nullptr;
  sp.final_r = final_r;
  sp.final_i = final_i;
  sp.M = M;
  sp.Mp = M;
  sp.chunks = chunks;
  sp.span = (chunks + kScanSpans - 1) / kScanSpans;
  sp.reverse = reverse;
  return launch_ex((const void*)mixer_carry_scan_kernel, dim3(kScanQ * ((M + 31) / 32), (unsigned)rows),
                   dim3(kScanThreads, 1, 1), kScanQ, 0, s, sp);
}

static int launch_error(cudaError_t e) {
  if (e == cudaSuccess) return SPARC_OK;
  set_err(cudaGetErrorString(e));
  return SPARC_ERR_LAUNCH;
}

// The kernels' mode from which optional inputs are given (-1: both a norm weight and projections).
static int fwd_mode(const SparcMixerFwdArgs* a) {
  if (a->projections != nullptr)
    return a->norm_weight != nullptr ? -1 : a->content_linear == 2 ? kModeScan : kModeProj;
  return a->norm_weight != nullptr ? kModeBlock : kModePlain;
}

// Validate the forward arguments and enqueue summary -> scan -> replay (scratch at `ws`).
static int run_forward(const SparcMixerFwdArgs* a, const Plan& pl, const WsLayout& L, char* ws, cudaStream_t s) {
  const bool proj = pl.mode == kModeProj || pl.mode == kModeScan;
  if (!a->x || !a->y || !a->carry || !a->controls || !a->nu_log || !a->theta_log ||
      (!proj && (!a->phase_direction || !a->radial_direction)) || !a->write_log_gain ||
      !a->write_phase_response || !a->write_radial_response) {
    set_err("null tensor pointer"); return SPARC_ERR_ARG;
  }
  if ((a->h0_r == nullptr) != (a->h0_i == nullptr) || (a->last_r == nullptr) != (a->last_i == nullptr)) {
    set_err("h0 / last pointers must be given in pairs"); return SPARC_ERR_ARG;
  }
  if (pl.mode == kModeBlock && (a->relu_mask == nullptr || !(a->norm_eps >= 0.0f))) {
    set_err("a block (norm_weight given) needs relu_mask and a non-negative norm_eps"); return SPARC_ERR_ARG;
  }
  FwdParams p;
  p.norm_w = a->norm_weight;
  p.norm_eps = a->norm_eps;
  p.mask = a->relu_mask;
  p.mask_words = pl.G * 16;
  p.x = a->x;
  p.y = a->y;
  p.pp = MixerParamPtrs{a->nu_log, a->theta_log, proj ? nullptr : a->phase_direction,
                        proj ? nullptr : a->radial_direction, a->write_log_gain, a->write_phase_response,
                        a->write_radial_response};
  p.proj_in = reinterpret_cast<const float2*>(a->projections);
  p.content_linear = a->content_linear;
  if (a->y_im != nullptr && pl.mode != kModeScan) {
    set_err("y_im is an output of the scan-level mode only"); return SPARC_ERR_ARG;
  }
  p.y_im = a->y_im;
  if (a->states != nullptr && proj) {
    set_err("states: in projection and scan-level mode the output y holds the states"); return SPARC_ERR_ARG;
  }
  p.states = a->states;
  p.h0_r = a->h0_r;
  p.h0_i = a->h0_i;
  p.ctl = reinterpret_cast<TokenCtl*>(a->controls);
  p.reset = a->reset;
  p.carry = reinterpret_cast<const float2*>(a->carry);
  p.agg = reinterpret_cast<float4*>(ws + L.agg);
  p.ls = reinterpret_cast<LaunchState*>(ws);
  p.B = a->batch;
  p.T = a->length;
  p.W = a->width;
  p.M = a->width / 2;
  p.Mp = pl.Mp;
  p.chunks = pl.chunks;
  p.tiles = pl.tiles;
  p.max_spin = a->max_spin ? a->max_spin : (1u << 20);
  p.use_tma = pl.tma && aligned16(a->x) && aligned16(a->controls) && aligned16(a->carry) &&
                      act_tensor_map(&p.map_x, a->x, a->dtype, p.B * p.T, p.M, p.W, pl.C) ? 1 : 0;
  const bool bf = a->dtype == SPARC_DTYPE_BF16;
  const void* ksum = bf ? Kernels<__nv_bfloat16>::sum(pl.mode) : Kernels<float>::sum(pl.mode);
  const void* krep = bf ? Kernels<__nv_bfloat16>::rep(pl.vec, pl.mode) : Kernels<float>::rep(pl.vec, pl.mode);
  int rc;
  {
    TimedLaunch tl(kTimeFwdSummary, s);
    rc = launch_error(launch_cluster(ksum, pl.G, kFwdThreads, pl.sum_clusters, pl.sum_smem, s, p));
  }
  if (rc != SPARC_OK) return rc;
  const ScanParams sp = scan_params(pl, L, ws, p.M, 0, a->h0_r, a->h0_i, a->last_r, a->last_i,
                                    reinterpret_cast<float2*>(a->carry));
  {
    TimedLaunch tl(kTimeFwdScan, s);
    rc = launch_error(launch_scan(pl, sp, s));
  }
  if (rc != SPARC_OK) return rc;
  TimedLaunch tl(kTimeFwdReplay, s);
  return launch_error(launch_plain(krep, dim3(pl.G, pl.rep_rows), kFwdThreads, pl.rep_smem, s, p));
}

}  // namespace sparc

using namespace sparc;

extern "C" {

const char* sparc_last_error(void) { return g_err; }

long long sparc_mixer_chunk_tokens(int dtype) { return chunk_for(dtype); }

long long sparc_mixer_carry_chunks(long long length, int dtype) {
  const int C = chunk_for(dtype);
  return (length + C - 1) / C;
}

size_t sparc_mixer_workspace_bytes(long long batch, long long length, int width, int dtype) {
  // one size for every mode (their gradient kernels' occupancy may differ)
  size_t total = 0;
  for (int mode = kModePlain; mode <= kModeScan; ++mode) {
    Plan pl;
    if (make_plan(batch, length, width, dtype, mode, &pl) != SPARC_OK) return 0;
    total = std::max(total, ws_layout(pl, batch, width / 2).total);
  }
  return total;
}

int sparc_mixer_controls_floats(void) { return (int)(sizeof(TokenCtl) / sizeof(float)); }

size_t sparc_exchange_buffer_bytes(int world) {
  return world >= 1 && world <= kXchgMaxRanks ? xchg_buffer_bytes(world) : 0;
}

int sparc_mixer_mask_words(int width) {
  if (width <= 0 || width % 2) return 0;
  return ((width / 2 + kFwdModes - 1) / kFwdModes) * 16;
}

int sparc_mixer_forward(const SparcMixerFwdArgs* a, void* stream) {
  NvtxRange nvtx(__func__);
  if (a == nullptr) { set_err("null args"); return SPARC_ERR_ARG; }
  const int mode = fwd_mode(a);
  if (mode < 0) { set_err("norm_weight and projections exclude each other"); return SPARC_ERR_ARG; }
  Plan pl;
  const int rc = make_plan(a->batch, a->length, a->width, a->dtype, mode, &pl);
  if (rc != SPARC_OK) return rc;
  const WsLayout L = ws_layout(pl, a->batch, a->width / 2);
  if (a->workspace == nullptr || a->workspace_bytes < L.total) { set_err("workspace too small"); return SPARC_ERR_WORKSPACE; }
  return run_forward(a, pl, L, static_cast<char*>(a->workspace), static_cast<cudaStream_t>(stream));
}

int sparc_mixer_backward(const SparcMixerBwdArgs* a, void* stream) {
  NvtxRange nvtx(__func__);
  if (a == nullptr) { set_err("null args"); return SPARC_ERR_ARG; }
  Plan pl;
  const bool block = a->norm_weight != nullptr;
  const bool proj = a->grad_projections != nullptr;
  if (block && proj) { set_err("norm_weight and grad_projections exclude each other"); return SPARC_ERR_ARG; }
  const int mode = proj ? (a->content_linear == 2 ? kModeScan : kModeProj) : block ? kModeBlock : kModePlain;
  int rc = make_plan(a->batch, a->length, a->width, a->dtype, mode, &pl);
  if (rc != SPARC_OK) return rc;
  const WsLayout L = ws_layout(pl, a->batch, a->width / 2);
  if (a->workspace == nullptr || a->workspace_bytes < L.total) { set_err("workspace too small"); return SPARC_ERR_WORKSPACE; }
  if (block ? (a->relu_mask == nullptr || a->grad_norm_weight == nullptr)
            : (!proj && a->y == nullptr && a->states == nullptr)) {
    set_err(block ? "a block needs relu_mask and grad_norm_weight" : "the forward's output y (or its states) is needed");
    return SPARC_ERR_ARG;
  }
  if (!a->x || !a->dy || !a->dx || !a->carry || !a->controls || !a->grad_nu_log || !a->grad_theta_log ||
      (!proj && (!a->grad_phase_direction || !a->grad_radial_direction || !a->phase_direction ||
                 !a->radial_direction)) ||
      !a->grad_write_log_gain || !a->grad_energy_response || !a->grad_write_phase_response ||
      !a->grad_write_radial_response) {
    set_err("null tensor pointer"); return SPARC_ERR_ARG;
  }
  if ((a->h0_r == nullptr) != (a->h0_i == nullptr) || (a->grad_last_r == nullptr) != (a->grad_last_i == nullptr) ||
      (a->grad_h0_r == nullptr) != (a->grad_h0_i == nullptr)) {
    set_err("paired pointers must be given together"); return SPARC_ERR_ARG;
  }
  char* ws = static_cast<char*>(a->workspace);
  BwdParams p;
  p.x = a->x;
  p.y = a->states != nullptr ? a->states : a->y;  // (the relu mask: sign(h) = sign(y) where y > 0)
  p.dy = a->dy;
  p.dx = a->dx;
  p.states = a->states;
  p.pp = MixerParamPtrs{a->nu_log, a->theta_log, proj ? nullptr : a->phase_direction,
                        proj ? nullptr : a->radial_direction, a->write_log_gain, a->write_phase_response,
                        a->write_radial_response};
  p.dp_out = reinterpret_cast<float2*>(a->grad_projections);
  p.content_linear = a->content_linear;
  p.h0_r = a->h0_r;
  p.h0_i = a->h0_i;
  p.glast_r = a->grad_last_r;
  p.glast_i = a->grad_last_i;
  p.ctl = reinterpret_cast<const TokenCtl*>(a->controls);
  p.norm_w = a->norm_weight;
  p.mask = a->relu_mask;
  p.mask_words = pl.G * 16;
  p.carry = reinterpret_cast<const float2*>(a->carry);
  p.kout = reinterpret_cast<const float2*>(ws + L.kout);
  p.agg = reinterpret_cast<float4*>(ws + L.agg);
  p.part = reinterpret_cast<double*>(ws + L.part);
  p.ls = reinterpret_cast<LaunchState*>(ws);
  p.B = a->batch;
  p.T = a->length;
  p.W = a->width;
  p.M = a->width / 2;
  p.Mp = pl.Mp;
  p.chunks = pl.chunks;
  p.tiles = pl.tiles;
  p.max_spin = a->max_spin ? a->max_spin : (1u << 20);
  const long long rows = p.B * p.T;
  // (a block reads no y: its relu mask comes as bits; the projection mode has no relu)
  p.use_tma = pl.tma && aligned16(a->x) && aligned16(p.y) && aligned16(a->dy) && aligned16(a->controls) &&
                      aligned16(a->carry) && aligned16(a->relu_mask) &&
                      act_tensor_map(&p.map_x, a->x, a->dtype, rows, p.M, p.W, pl.C) &&
                      (block || proj || act_tensor_map(&p.map_y, p.y, a->dtype, rows, p.M, p.W, pl.C)) &&
                      act_tensor_map(&p.map_dy, a->dy, a->dtype, rows, p.M, p.W, pl.C) ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf = a->dtype == SPARC_DTYPE_BF16;
  const void* krsum = bf ? Kernels<__nv_bfloat16>::rsum(pl.mode) : Kernels<float>::rsum(pl.mode);
  const void* kgrad = bf ? Kernels<__nv_bfloat16>::grad(pl.vec, pl.mode) : Kernels<float>::grad(pl.vec, pl.mode);
  // With the forward's states (and tensor maps) the gradient kernel reads them in half-tile
  // stages instead of replaying the recurrence; its maps have boxes of C/2 (C/2 + 1) rows.
  const void* ksaved = bf ? Kernels<__nv_bfloat16>::saved(pl.vec, pl.mode, pl.G) : Kernels<float>::saved(pl.vec, pl.mode, pl.G);
  const int part = pl.C / Kernels<float>::saved_split(pl.G);  // tokens per stage
  BwdParams ps = p;
  const bool saved = ksaved != nullptr && a->states != nullptr && p.use_tma && aligned16(a->states) &&
                     act_tensor_map(&ps.map_x, a->x, a->dtype, rows, p.M, p.W, part) &&
                     act_tensor_map(&ps.map_dy, a->dy, a->dtype, rows, p.M, p.W, part) &&
                     act_tensor_map(&ps.map_h, a->states, a->dtype, rows, p.M, p.W, part + 1);
  {
    TimedLaunch tl(kTimeBwdSummary, s);
    rc = launch_error(launch_plain(krsum, dim3(pl.G, pl.rsum_rows), kBwdThreads, pl.rsum_smem, s, p));
  }
  if (rc != SPARC_OK) return rc;
  const ScanParams sp = scan_params(pl, L, ws, p.M, 1, a->grad_last_r, a->grad_last_i, a->grad_h0_r,
                                    a->grad_h0_i, reinterpret_cast<float2*>(ws + L.kout));
  {
    TimedLaunch tl(kTimeBwdScan, s);
    rc = launch_error(launch_scan(pl, sp, s));
  }
  if (rc != SPARC_OK) return rc;
  {
    TimedLaunch tl(kTimeBwdGrad, s);
    rc = launch_error(saved ? launch_cluster(ksaved, pl.G, kGradThreads, pl.saved_clusters, pl.saved_smem, s, ps)
                            : launch_cluster(kgrad, pl.G, kGradThreads, pl.grad_clusters, pl.grad_smem, s, p));
  }
  if (rc != SPARC_OK) return rc;
  ReduceParams r;
  r.part = p.part;
  r.clusters = saved ? pl.saved_clusters : pl.grad_clusters;
  r.Mp = pl.Mp;
  r.M = p.M;
  r.W = p.W;
  r.theta_log = a->theta_log;
  r.g_nu_log = a->grad_nu_log;
  r.g_theta_log = a->grad_theta_log;
  r.g_wlg = a->grad_write_log_gain;
  r.g_wpr = a->grad_write_phase_response;
  r.g_wrr = a->grad_write_radial_response;
  r.g_energy = a->grad_energy_response;
  r.g_phase_dir = proj ? nullptr : a->grad_phase_direction;
  r.g_radial_dir = proj ? nullptr : a->grad_radial_direction;
  r.g_norm_w = block ? a->grad_norm_weight : nullptr;
  r.xchg = PeerExchange{};
  r.xchg.world = a->exchange_world > 1 ? a->exchange_world : 1;
  if (r.xchg.world > 1) {
    if (r.xchg.world > kXchgMaxRanks || a->exchange_rank < 0 || a->exchange_rank >= r.xchg.world ||
        a->exchange_status == nullptr) {
      set_err("exchange_world must be 2..8 with a rank in [0, world) and a status word");
      return SPARC_ERR_ARG;
    }
    if ((long long)((pl.Mp + 31) / 32) * (kPartModes + 1) > kXchgSlots) {
      set_err("width too large for the gradient exchange's slots");
      return SPARC_ERR_SHAPE;
    }
    for (int i = 0; i < r.xchg.world; ++i) {
      if (a->exchange_buffers[i] == nullptr) { set_err("null exchange buffer"); return SPARC_ERR_ARG; }
      r.xchg.base[i] = static_cast<unsigned char*>(a->exchange_buffers[i]);
    }
    r.xchg.rank = a->exchange_rank;
    r.xchg.status = a->exchange_status;
    r.xchg.max_spin = 1u << 24;
  }
  TimedLaunch tl(kTimeBwdReduce, s);
  return launch_error(launch_ex((const void*)mixer_reduce_kernel, dim3((pl.Mp + 31) / 32, kPartModes + 1),
                               dim3(32, kReduceWarps), 0, 0, s, r));
}

// ------------------------------------------------------------------------------ no-alloc variant
// sparc_mixer_forward_noalloc: the same forward launches, with their scratch (launch counters,
// scan flags, segment and chunk aggregates) in a fixed array that lives in the library itself,
// for callers that cannot allocate device memory. See the declaration in sparc_b200.h.
}  // extern "C"

namespace sparc {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB per GPU, held until exit

// Zero-initialised when the library's module is loaded on a device. Host code must not use
// this name as a device address: noalloc_scratch() looks the address up per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static void* noalloc_scratch(int dev) {
  static std::mutex mu;
  static void* addr[64] = {};
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* ptr = nullptr;
    // the current device is `dev`: the lookup (and the lazy module load it may trigger) binds
    // the array of this device
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) {
      cudaGetLastError();
      return nullptr;
    }
    addr[dev] = ptr;
  }
  return addr[dev];
}

}  // namespace sparc

extern "C" {

size_t sparc_mixer_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int sparc_mixer_forward_noalloc(const SparcMixerFwdArgs* a, void* stream) {
  NvtxRange nvtx(__func__);
  if (a == nullptr) { set_err("null args"); return SPARC_ERR_ARG; }
  const int mode = fwd_mode(a);
  if (mode < 0) { set_err("norm_weight and projections exclude each other"); return SPARC_ERR_ARG; }
  Plan pl;
  const int rc = make_plan(a->batch, a->length, a->width, a->dtype, mode, &pl);
  if (rc != SPARC_OK) return rc;
  const WsLayout L = ws_layout(pl, a->batch, a->width / 2);
  // the forward uses the launch state, the scan's flags and segment arrays, and the chunk
  // aggregates (everything before the backward's adjoint carries)
  const size_t need = L.kout;
  if (need > kNoAllocScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "sparc_mixer_forward_noalloc: batch %lld x length %lld x width %d needs %zu bytes of "
             "scratch, above the built-in %zu; use sparc_mixer_forward with a workspace",
             a->batch, a->length, a->width, need, kNoAllocScratchBytes);
    set_err(msg);
    return SPARC_ERR_WORKSPACE;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); set_err("no current CUDA device"); return SPARC_ERR_LAUNCH; }
  char* ws = static_cast<char*>(noalloc_scratch(dev));
  if (ws == nullptr) { set_err("cudaGetSymbolAddress failed for the built-in scratch"); return SPARC_ERR_LAUNCH; }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return run_forward(a, pl, L, ws, s);
}

size_t sparc_mixer_noalloc_scratch_needed(long long batch, long long length, int width, int dtype) {
  // the largest forward scratch over the three modes (plain, block, projection)
  size_t need = 0;
  for (int mode = kModePlain; mode <= kModeScan; ++mode) {
    Plan pl;
    if (make_plan(batch, length, width, dtype, mode, &pl) != SPARC_OK) return 0;
    need = std::max(need, ws_layout(pl, batch, width / 2).kout);
  }
  return need;
}

int sparc_mixer_noalloc_read_status(unsigned* status, void* stream) {
  if (status == nullptr) { set_err("null pointer"); return SPARC_ERR_ARG; }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); set_err("no current CUDA device"); return SPARC_ERR_LAUNCH; }
  const void* ws = noalloc_scratch(dev);
  if (ws == nullptr) { set_err("cudaGetSymbolAddress failed for the built-in scratch"); return SPARC_ERR_LAUNCH; }
  return sparc_read_status(ws, status, stream);
}

int sparc_mixer_noalloc_clear_status(void* stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); set_err("no current CUDA device"); return SPARC_ERR_LAUNCH; }
  void* ws = noalloc_scratch(dev);
  if (ws == nullptr) { set_err("cudaGetSymbolAddress failed for the built-in scratch"); return SPARC_ERR_LAUNCH; }
  return sparc_clear_status(ws, stream);
}

int sparc_read_status(const void* workspace, unsigned* status, void* stream) {
  if (workspace == nullptr || status == nullptr) { set_err("null pointer"); return SPARC_ERR_ARG; }
  const LaunchState* ls = static_cast<const LaunchState*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(status, &ls->status, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) { set_err(cudaGetErrorString(e)); return SPARC_ERR_LAUNCH; }
  return SPARC_OK;
}

int sparc_clear_status(void* workspace, void* stream) {
  if (workspace == nullptr) { set_err("null pointer"); return SPARC_ERR_ARG; }
  LaunchState* ls = static_cast<LaunchState*>(workspace);
  cudaError_t e = cudaMemsetAsync(&ls->status, 0, sizeof(unsigned), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) { set_err(cudaGetErrorString(e)); return SPARC_ERR_LAUNCH; }
  return SPARC_OK;
}

}  // extern "C"
