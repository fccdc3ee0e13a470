// Fused single-step SPARC decode for B200 (sm_100a).
//
// One CTA of 512 threads per batch row: the controller projection needs the whole row (a block
// reduction over `width` columns), then every thread updates its modes (up to four; widths up to
// 4096). Everything a thread needs that does not depend on the token's controls is loaded and
// computed first, in flight with the projection: its x values for the write, its old state and
// its modes' constants (e^nu_log, the rotation e^{i theta}, the write gain's constant part), so
// after the block reduction only the control-dependent arithmetic remains. Launches carry the
// programmatic-stream-serialisation attribute, so a step's launch overlaps the previous step's
// tail (pdl_wait comes first: the previous kernel may write x, the state or the parameters).
// Parity target: _latest_sparc_decode, forward/decode.py:11-55 (Botwwt/sparc). Decode is
// latency-bound (a few KB per row), so the accurate libm functions are used throughout.
#include "common.cuh"
#include "sparc_b200.h"
#include "timing.cuh"

namespace sparc {

constexpr int kDecodeThreads = 512;
constexpr int kDecodeModes = 4;  // modes per thread at most (M <= 2048)

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
  pdl_wait();
  const long long b = blockIdx.x;
  const int W = p.W, M = p.M;
  const int tid = threadIdx.x;
  const TIO* xrow = static_cast<const TIO*>(p.x) + b * W;

  // control-independent work first: the thread's modes' x values, old states and constants
  float xr[kDecodeModes], xi[kDecodeModes], hr[kDecodeModes], hi[kDecodeModes];
  float nu[kDecodeModes], ct[kDecodeModes], st[kDecodeModes], gconst[kDecodeModes], den[kDecodeModes];
  float wpr[kDecodeModes], wrr[kDecodeModes];
#pragma unroll
  for (int j = 0; j < kDecodeModes; ++j) {
    const int m = tid + j * kDecodeThreads;
    if (m < M) {
      xr[j] = Io<TIO>::load(xrow + m);
      xi[j] = Io<TIO>::load(xrow + M + m);
      hr[j] = p.state_r[b * M + m];
      hi[j] = p.state_i[b * M + m];
      nu[j] = expf(p.nu_log[m]);
      sincosf(expf(p.theta_log[m]), &st[j], &ct[j]);
      den[j] = expm1f(-2.0f * nu[j]);
      gconst[j] = expf(p.wlg[m]);
      wpr[j] = p.wpr[m];
      wrr[j] = p.wrr[m];
    }
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
      const float tau0 = tanhf(t0 + p.phase_dir[W]);
      const float tau1 = tanhf(t1 + p.radial_dir[W]);
      ctl[0] = tau0;
      ctl[1] = tau1;
      ctl[2] = kHalfPi * tau0;      // delta
      ctl[3] = expf(kLn16 * tau1);  // e^eta
    }
  }
  __syncthreads();
  const float tau0 = ctl[0], tau1 = ctl[1], delta = ctl[2], E = ctl[3];
  TIO* yrow = static_cast<TIO*>(p.y) + b * W;
#pragma unroll
  for (int j = 0; j < kDecodeModes; ++j) {
    const int m = tid + j * kDecodeThreads;
    if (m < M) {
      const float z = nu[j] * E;
      const float rho = expf(-z);
      float s, c;
      sincosf((1.0f - rho) * delta, &s, &c);  // rotate e^{i theta} by the token's phase offset
      const float pc = ct[j] * c - st[j] * s, ps = st[j] * c + ct[j] * s;
      const float ratio = sqrtf(expm1f(-2.0f * z) / den[j]);
      const float q = tau0 * wpr[j] + tau1 * wrr[j];
      const float gate = 2.0f / (1.0f + expf(-q));
      const float gain = gconst[j] * ratio * gate;
      const float ar = rho * pc, ai = rho * ps;
      const float nr = fmaf(ar, hr[j], fmaf(-ai, hi[j], gain * tanhf(xr[j])));
      const float ni = fmaf(ai, hr[j], fmaf(ar, hi[j], gain * tanhf(xi[j])));
      p.new_r[b * M + m] = nr;
      p.new_i[b * M + m] = ni;
      Io<TIO>::store(yrow + m, fmaxf(nr, 0.0f));
      Io<TIO>::store(yrow + M + m, fmaxf(ni, 0.0f));
    }
  }
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
  if (a->width / 2 > kDecodeThreads * kDecodeModes) return fail(SPARC_ERR_SHAPE, "width above the decode kernel's limit");
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
  cfg.gridDim = dim3((unsigned)a->batch, 1, 1);
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
