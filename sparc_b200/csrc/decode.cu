// Fused single-step SPARC decode for B200 (sm_100a).
//
// One CTA per batch row: the controller projection needs the whole row (a block reduction
// over `width` columns), then every thread updates its modes. Parity target:
// _latest_sparc_decode, forward/decode.py:11-55 (Botwwt/sparc). Decode is latency-bound
// (a few KB per row), so the accurate libm functions are used throughout.
#include "common.cuh"
#include "sparc_b200.h"
#include "timing.cuh"

namespace sparc {

constexpr int kDecodeThreads = 256;

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

template <typename TIO>
__global__ void __launch_bounds__(kDecodeThreads) decode_kernel(const DecodeParams p) {
  const long long b = blockIdx.x;
  const int W = p.W, M = p.M;
  const TIO* xrow = static_cast<const TIO*>(p.x) + b * W;
  float s0 = 0.0f, s1 = 0.0f;
  for (int c = threadIdx.x; c < W; c += kDecodeThreads) {
    const float xv = Io<TIO>::load(xrow + c);
    s0 = fmaf(xv, p.phase_dir[c], s0);
    s1 = fmaf(xv, p.radial_dir[c], s1);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    s0 += __shfl_xor_sync(0xffffffffu, s0, o);
    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
  }
  __shared__ float red[2][kDecodeThreads / 32];
  __shared__ float ctl[4];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    red[0][warp] = s0;
    red[1][warp] = s1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float t0 = 0.0f, t1 = 0.0f;
    for (int w = 0; w < kDecodeThreads / 32; ++w) {
      t0 += red[0][w];
      t1 += red[1][w];
    }
    const float tau0 = tanhf(t0 + p.phase_dir[W]);
    const float tau1 = tanhf(t1 + p.radial_dir[W]);
    ctl[0] = tau0;
    ctl[1] = tau1;
    ctl[2] = kHalfPi * tau0;       // delta
    ctl[3] = expf(kLn16 * tau1);   // e^eta
  }
  __syncthreads();
  const float tau0 = ctl[0], tau1 = ctl[1], delta = ctl[2], E = ctl[3];
  TIO* yrow = static_cast<TIO*>(p.y) + b * W;
  for (int m = threadIdx.x; m < M; m += kDecodeThreads) {
    const float nu = expf(p.nu_log[m]);
    const float theta = expf(p.theta_log[m]);
    const float z = nu * E;
    const float rho = expf(-z);
    float s, c;
    sincosf(theta + (1.0f - rho) * delta, &s, &c);
    const float ratio = sqrtf(expm1f(-2.0f * z) / expm1f(-2.0f * nu));
    const float q = tau0 * p.wpr[m] + tau1 * p.wrr[m];
    const float gate = 2.0f / (1.0f + expf(-q));
    const float gain = expf(p.wlg[m]) * ratio * gate;
    const float cr = tanhf(Io<TIO>::load(xrow + m));
    const float ci = tanhf(Io<TIO>::load(xrow + M + m));
    const float hr = p.state_r[b * M + m], hi = p.state_i[b * M + m];
    const float ar = rho * c, ai = rho * s;
    const float nr = fmaf(ar, hr, fmaf(-ai, hi, gain * cr));
    const float ni = fmaf(ai, hr, fmaf(ar, hi, gain * ci));
    p.new_r[b * M + m] = nr;
    p.new_i[b * M + m] = ni;
    Io<TIO>::store(yrow + m, fmaxf(nr, 0.0f));
    Io<TIO>::store(yrow + M + m, fmaxf(ni, 0.0f));
  }
}

}  // namespace sparc

using namespace sparc;

extern "C" int sparc_decode_step(const SparcDecodeArgs* a, void* stream) {
  if (a == nullptr || !a->x || !a->y || !a->state_r || !a->state_i || !a->new_state_r ||
      !a->new_state_i || !a->nu_log || !a->theta_log || !a->phase_direction ||
      !a->radial_direction || !a->write_log_gain || !a->write_phase_response ||
      !a->write_radial_response) {
    return SPARC_ERR_ARG;
  }
  if (a->batch <= 0 || a->width <= 0 || (a->width % 2) != 0 || a->batch > 0x7fffffffLL) return SPARC_ERR_SHAPE;
  if (a->new_state_r == a->state_r || a->new_state_i == a->state_i) return SPARC_ERR_ARG;
  DecodeParams p{a->x, a->y, a->state_r, a->state_i, a->new_state_r, a->new_state_i,
                 a->nu_log, a->theta_log, a->phase_direction, a->radial_direction,
                 a->write_log_gain, a->write_phase_response, a->write_radial_response,
                 a->width, a->width / 2};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  TimedLaunch tl(kTimeDecode, s);
  if (a->dtype == SPARC_DTYPE_BF16) {
    decode_kernel<__nv_bfloat16><<<(unsigned)a->batch, kDecodeThreads, 0, s>>>(p);
  } else if (a->dtype == SPARC_DTYPE_F32) {
    decode_kernel<float><<<(unsigned)a->batch, kDecodeThreads, 0, s>>>(p);
  } else {
    return SPARC_ERR_DTYPE;
  }
  return cudaGetLastError() == cudaSuccess ? SPARC_OK : SPARC_ERR_LAUNCH;
}
