// Fused single-step SPARC decode for B200 (sm_100a).
//
// Grid (batch, S) of 512-thread CTAs, S = ceil(M / 512): CTA (b, s) updates modes
// [512 s, 512 s + 512) of batch row b, one mode per thread, so that more CTAs share a step's
// short latency chain. The controller projection needs the whole row: every CTA of the row
// computes it (a block reduction over `width` columns; the row is a few KB in L2) instead of
// exchanging it. Everything a thread needs that does not depend on the token's controls is
// loaded and computed first, in flight with the projection: its x values for the write, its old
// state and its mode's constants (e^nu_log, the rotation e^{i theta}, the write gain's constant
// part), so after the reduction only the control-dependent arithmetic remains, in the same
// approximations as the sequence kernels (hardware exp2 / reciprocal / square root, the series
// of the bounded phase offset and of 1 - e^{-2z} for small z, tanh as 1 - 2 / (e^{2x} + 1)): the
// decode trajectory follows the sequence scan to rounding. Launches carry the
// programmatic-stream-serialisation attribute, so a step's launch overlaps the previous step's
// tail (pdl_wait comes first: the previous kernel may write x, the state or the parameters).
// Parity target: _latest_sparc_decode, forward/decode.py:11-55 (Botwwt/sparc).
#include "common.cuh"
#include "sparc_b200.h"
#include "timing.cuh"

namespace sparc {

constexpr int kDecodeThreads = 512;
constexpr int kDecodeMaxSplit = 4;  // CTAs per row at most (M <= 2048)

struct DecodeParams {
  const void* x;
  void* y;
  const float* state_r;
  const float* state_i;
  float* new_r;
  float* new_i;
  const float* nu_log;
  const float* theta_log;
  const float* phase_dir;
  const float* radial_dir;
  const float* wlg;
  const float* wpr;
  const float* wrr;
  int W, M;
};

__device__ __forceinline__ float tanh_exp(float x) { return fmaf(-2.0f, rcp_approx(ex2_approx(2.0f * kLog2e * x) + 1.0f), 1.0f); }

template <typename TIO>
__global__ void __launch_bounds__(kDecodeThreads) decode_kernel(const DecodeParams p) {
  pdl_wait();
  const long long b = blockIdx.x;
  const int W = p.W, M = p.M;
  const int tid = threadIdx.x;
  const int m = blockIdx.y * kDecodeThreads + tid;
  const bool act = m < M;
  const TIO* xrow = static_cast<const TIO*>(p.x) + b * W;

  // control-independent work first: the mode's x values, old state and constants
  float xr = 0.0f, xi = 0.0f, hr = 0.0f, hi = 0.0f, nu = 0.0f, ct = 1.0f, st = 0.0f, gconst = 0.0f, iden = 0.0f;
  float wpr = 0.0f, wrr = 0.0f;
  if (act) {
    xr = Io<TIO>::load(xrow + m);
    xi = Io<TIO>::load(xrow + M + m);
    hr = p.state_r[b * M + m];
    hi = p.state_i[b * M + m];
    nu = expf(p.nu_log[m]);
    sincosf(expf(p.theta_log[m]), &st, &ct);
    iden = 1.0f / -expm1f(-2.0f * nu);
    gconst = expf(p.wlg[m]);
    wpr = p.wpr[m];
    wrr = p.wrr[m];
  }

  // controller projection of the row
  float s0 = 0.0f, s1 = 0.0f;
  for (int c = tid; c < W; c += kDecodeThreads) {
    const float xv = Io<TIO>::load(xrow + c);
    s0 = fmaf(xv, p.phase_dir[c], s0);
    s1 = fmaf(xv, p.radial_dir[c], s1);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    s0 += __shfl_xor_sync(0xffffffffu, s0, o);
    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
  }
  constexpr int NW = kDecodeThreads / 32;
  __shared__ float red[2][NW];
  __shared__ float ctl[4];
  const int lane = tid & 31, warp = tid >> 5;
  if (lane == 0) {
    red[0][warp] = s0;
    red[1][warp] = s1;
  }
  __syncthreads();
  if (warp == 0) {
    // warp 0 sums the warps' partials in a fixed order, lane 0 computes the controls
    float t0 = lane < NW ? red[0][lane] : 0.0f;
    float t1 = lane < NW ? red[1][lane] : 0.0f;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      t0 += __shfl_xor_sync(0xffffffffu, t0, o);
      t1 += __shfl_xor_sync(0xffffffffu, t1, o);
    }
    if (lane == 0) {
      const float tau0 = tanh_accurate(t0 + p.phase_dir[W]);
      const float tau1 = tanh_accurate(t1 + p.radial_dir[W]);
      ctl[0] = tau0;
      ctl[1] = tau1;
      ctl[2] = kHalfPi * tau0;      // delta
      ctl[3] = expf(kLn16 * tau1);  // e^eta
    }
  }
  __syncthreads();
  if (!act) return;
  const float tau0 = ctl[0], tau1 = ctl[1], delta = ctl[2], E = ctl[3];
  const float z = nu * E;
  const float rho = ex2_approx(-kLog2e * z);
  float s, c;
  sincos_halfpi(fmaf(-rho, delta, delta), &s, &c);  // rotate e^{i theta} by (1 - rho) delta, |.| <= pi/2
  const float pc = ct * c - st * s, ps = st * c + ct * s;
  // 1 - e^{-2z}: its series below u = 2z = 1/4 (no cancellation), else 1 - rho^2
  const float u = 2.0f * z;
  const float ser = u * fmaf(fmaf(fmaf(fmaf(fmaf(-1.3888888888888889e-3f, u, 8.3333333333333333e-3f), u,
                                           -4.1666666666666667e-2f), u, 1.6666666666666667e-1f), u, -0.5f), u, 1.0f);
  const float num = u < 0.25f ? ser : fmaf(-rho, rho, 1.0f);
  const float q = fmaf(tau0, wpr, tau1 * wrr);
  const float gate = 2.0f * rcp_approx(1.0f + ex2_approx(-kLog2e * q));
  const float gain = gconst * sqrt_approx(num * iden) * gate;
  const float ar = rho * pc, ai = rho * ps;
  const float nr = fmaf(ar, hr, fmaf(-ai, hi, gain * tanh_exp(xr)));
  const float ni = fmaf(ai, hr, fmaf(ar, hi, gain * tanh_exp(xi)));
  p.new_r[b * M + m] = nr;
  p.new_i[b * M + m] = ni;
  TIO* yrow = static_cast<TIO*>(p.y) + b * W;
  Io<TIO>::store(yrow + m, fmaxf(nr, 0.0f));
  Io<TIO>::store(yrow + M + m, fmaxf(ni, 0.0f));
}

}  // namespace sparc

using namespace sparc;

extern "C" int sparc_decode_step(const SparcDecodeArgs* a, void* stream) {
  NvtxRange nvtx(__func__);
  if (a == nullptr) return fail(SPARC_ERR_ARG, "null args");
  if (!a->x || !a->y || !a->state_r || !a->state_i || !a->new_state_r || !a->new_state_i || !a->nu_log ||
      !a->theta_log || !a->phase_direction || !a->radial_direction || !a->write_log_gain ||
      !a->write_phase_response || !a->write_radial_response) {
    return fail(SPARC_ERR_ARG, "null tensor pointer");
  }
  if (a->batch <= 0 || a->width <= 0 || a->batch > 0x7fffffffLL)
    return fail(SPARC_ERR_SHAPE, "batch and width must be positive");
  if (a->width % 2) return fail(SPARC_ERR_SHAPE, "SPARC rnn_width must be even");
  if (a->width / 2 > kDecodeThreads * kDecodeMaxSplit) return fail(SPARC_ERR_SHAPE, "width above the decode kernel's limit");
  if (a->new_state_r == a->state_r || a->new_state_i == a->state_i)
    return fail(SPARC_ERR_ARG, "the new state must not alias the old one");
  if (a->dtype != SPARC_DTYPE_BF16 && a->dtype != SPARC_DTYPE_F32) return fail(SPARC_ERR_DTYPE, "unsupported dtype");
  DecodeParams p{a->x, a->y, a->state_r, a->state_i, a->new_state_r, a->new_state_i,
                 a->nu_log, a->theta_log, a->phase_direction, a->radial_direction,
                 a->write_log_gain, a->write_phase_response, a->write_radial_response,
                 a->width, a->width / 2};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  TimedLaunch tl(kTimeDecode, s);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a->batch, (unsigned)((a->width / 2 + kDecodeThreads - 1) / kDecodeThreads), 1);
  cfg.blockDim = dim3(kDecodeThreads, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {&p};
  const void* k = a->dtype == SPARC_DTYPE_BF16 ? (const void*)decode_kernel<__nv_bfloat16> : (const void*)decode_kernel<float>;
  const cudaError_t e = cudaLaunchKernelExC(&cfg, k, args);
  return e == cudaSuccess ? SPARC_OK : fail(SPARC_ERR_LAUNCH, cudaGetErrorString(e));
}
