// RTRL online traces of the SPARC cell for B200 (sm_100a): the forward-mode trace update and the
// trace-based gradients of sparc-impl/sparc/training/rtrl.py (_trace_step 154-201,
// _stored_rtrl_backward 220-240).
//
// Every recurrent parameter has a complex trace per batch row: the five modal vectors [B, M],
// content_real / content_imag [B, W, M] and the two controllers [B, W+1, M] (W = input size).
// One step advances every trace as trace' = a (keep ? trace : 0) + direct, with a the step's
// transition and direct the step's own derivative of h' = a h + gain c (the closed forms are in
// rtrl_coef). The content and controller traces are rank-one updates over the inputs
// (direct = x_j * d_m), so the step is a stream over the traces: each thread owns one mode m of
// one batch row, computes the row's coefficients once in registers and walks a slab of the
// trace rows j with coalesced 8-byte loads and stores (consecutive threads, consecutive modes).
// The content products u = x content and the controller projections p = [x, 1] controller are
// the caller's matrix products (inputs here), so the step kernel is elementwise in (b, m) and
// HBM-bound on the traces: 64 bytes per (b, j, m) (four traces read and written).
//
// The gradient of a loss on h' (g_r = dL/dRe h', g_i = dL/dIm h'; JAX's cotangent is
// g_r - i g_i) w.r.t. a parameter is g_r Re(trace) + g_i Im(trace) summed over the batch (and
// over the modes for the controllers), read from the step's new traces; the input side returns
// the gradients of u and p (the caller finishes x's). All sums run in a fixed order: one CTA per
// trace row j (content and controller gradients), per batch row (projection gradients) and per
// 128 modes (modal gradients).
#include "common.cuh"
#include "sparc_b200.h"
#include "timing.cuh"

#include <algorithm>
#include <cstdio>

namespace sparc {

constexpr int kRtrlThreads = 128;  // one mode per thread
constexpr int kRtrlUnroll = 4;     // trace rows in flight per thread
constexpr int kRtrlSavedFloats = 8;
constexpr int kRtrlGradThreads = 256;
static_assert(kRtrlUnroll == 4, "the gradient kernel combines four partial sums");

struct RtrlStepParams {
  const float* x;
  const float* u;       // [B, 2M]
  const float2* proj;   // [B]
  const unsigned char* reset;
  const float2* state;
  float2* new_state;
  const float* dlog;
  const float* flog;
  const float* wlg;
  const float* wpr;
  const float* wrr;
  const float2* tr[9];
  float2* ntr[9];
  float4* saved;        // [B, M, 2]
  long long B;
  int W, M, lin, rows_per_z;
};

struct RtrlCoef {
  float2 a;
  float gsr, gsi;  // gain * content slope
  float2 d[5];     // modal directs
  float2 dph, dret;
  float2 hnew;
};

__device__ __forceinline__ float2 cmulf(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

// The step's transition, write and the forward-mode derivative of h' = a h + gain c w.r.t. each
// parameter (rtrl.py:61-108; recurrence.py:28-63 for the terms). With z = nu e^eta,
// rho = e^-z, s0 = 1 - tanh(p0)^2, s1 = 1 - tanh(p1)^2, dyn = z e^-2z / -expm1(-2z),
// stat = nu e^-2nu / -expm1(-2nu), gq = gain (1 - gate / 2):
//   decay_log:  z (i rho delta - 1) a h + gain (dyn - stat) c      frequency_log: i theta a h
//   write_log_gain: gain c   write_phase_response: gq tau0 c   write_retention_response: gq tau1 c
//   phase_controller (bias entry): i (1 - rho)(pi/2) s0 a h + gq wpr s0 c
//   retention_controller (bias entry): ln16 s1 z (i rho delta - 1) a h + (gain dyn ln16 + gq wrr) s1 c
//   content_real[j] / content_imag[j]: x_j gain slope_r / i x_j gain slope_i
// (slope = 1 - tanh(u)^2, or 1 for a linear content); controller entry j is x_j times its bias
// entry's direct (x_W = 1).
// Latency- or HBM-bound work: the accurate libm functions are used throughout.
__device__ __forceinline__ RtrlCoef rtrl_coef(const RtrlStepParams& p, long long b, int m, bool keep) {
  RtrlCoef k;
  const int M = p.M;
  const float ur = p.u[b * 2 * M + m], ui = p.u[b * 2 * M + M + m];
  const float2 pj = p.proj[b];
  const float2 h = keep ? p.state[b * M + m] : make_float2(0.0f, 0.0f);
  const float nu = expf(p.dlog[m]), theta = expf(p.flog[m]);
  const float tau0 = tanhf(pj.x), tau1 = tanhf(pj.y);
  const float delta = kHalfPi * tau0, E = expf(kLn16 * tau1);
  const float z = nu * E, rho = expf(-z);
  float sn, cs;
  sincosf(theta + (1.0f - rho) * delta, &sn, &cs);
  k.a = make_float2(rho * cs, rho * sn);
  const float num = -expm1f(-2.0f * z), den = -expm1f(-2.0f * nu);
  const float wpr = p.wpr[m], wrr = p.wrr[m];
  const float gate = 2.0f / (1.0f + expf(-(tau0 * wpr + tau1 * wrr)));
  const float gain = expf(p.wlg[m]) * sqrtf(num / den) * gate;
  const float cr = p.lin ? ur : tanhf(ur), ci = p.lin ? ui : tanhf(ui);
  const float sr = p.lin ? 1.0f : 1.0f - cr * cr, si = p.lin ? 1.0f : 1.0f - ci * ci;
  const float dyn = z * expf(-2.0f * z) / num, stat = nu * expf(-2.0f * nu) / den;
  const float gq = gain * (1.0f - 0.5f * gate);
  const float s0 = 1.0f - tau0 * tau0, s1 = 1.0f - tau1 * tau1;
  const float2 ah = cmulf(k.a, h);
  const float2 c = make_float2(cr, ci);
  // (i rho delta - 1) a h
  const float2 rot = make_float2(-ah.x - rho * delta * ah.y, -ah.y + rho * delta * ah.x);
  const float wd = gain * (dyn - stat);
  k.d[0] = make_float2(z * rot.x + wd * c.x, z * rot.y + wd * c.y);
  k.d[1] = make_float2(-theta * ah.y, theta * ah.x);
  k.d[2] = make_float2(gain * c.x, gain * c.y);
  k.d[3] = make_float2(gq * tau0 * c.x, gq * tau0 * c.y);
  k.d[4] = make_float2(gq * tau1 * c.x, gq * tau1 * c.y);
  const float ph = (1.0f - rho) * kHalfPi * s0, wph = gq * wpr * s0;
  k.dph = make_float2(-ph * ah.y + wph * c.x, ph * ah.x + wph * c.y);
  const float rz = z * kLn16 * s1, wrt = (gain * dyn * kLn16 + gq * wrr) * s1;
  k.dret = make_float2(rz * rot.x + wrt * c.x, rz * rot.y + wrt * c.y);
  k.gsr = gain * sr;
  k.gsi = gain * si;
  k.hnew = make_float2(ah.x + gain * c.x, ah.y + gain * c.y);
  return k;
}

// grid (ceil(M / 128), B, Z): blockIdx.z takes the trace rows [z R, z R + R) of the W + 1
// (R = rows_per_z); z == 0 also writes the new state, the modal traces and the saved values.
__global__ void __launch_bounds__(kRtrlThreads) rtrl_step_kernel(const __grid_constant__ RtrlStepParams p) {
  pdl_wait();
  const int m = blockIdx.x * kRtrlThreads + threadIdx.x;
  const long long b = blockIdx.y;
  const int M = p.M, W = p.W;
  if (m >= M) return;  // (no block-level synchronisation below)
  const bool keep = p.reset == nullptr || p.reset[b] == 0;
  const RtrlCoef k = rtrl_coef(p, b, m, keep);
  const long long bm = b * M + m;
  auto adv = [&](float2 t, float2 d) {  // a (keep ? t : 0) + d
    if (!keep) t = make_float2(0.0f, 0.0f);
    return make_float2(fmaf(k.a.x, t.x, fmaf(-k.a.y, t.y, d.x)), fmaf(k.a.x, t.y, fmaf(k.a.y, t.x, d.y)));
  };
  if (blockIdx.z == 0) {
    p.new_state[bm] = k.hnew;
#pragma unroll
    for (int q = 0; q < 5; ++q) p.ntr[q][bm] = adv(p.tr[q][bm], k.d[q]);
    p.saved[bm * 2] = make_float4(k.gsr, k.gsi, k.dph.x, k.dph.y);
    p.saved[bm * 2 + 1] = make_float4(k.dret.x, k.dret.y, 0.0f, 0.0f);
  }
  const int j0 = blockIdx.z * p.rows_per_z;
  const int j1 = min(W + 1, j0 + p.rows_per_z);
  const float* xb = p.x + b * W;
  const long long cbase = b * (long long)W * M + m;         // content traces [B, W, M]
  const long long kbase = b * (long long)(W + 1) * M + m;   // controller traces [B, W+1, M]
  for (int j = j0; j < j1; j += kRtrlUnroll) {
    float2 tc[kRtrlUnroll][4];
    float xj[kRtrlUnroll];
#pragma unroll
    for (int u = 0; u < kRtrlUnroll; ++u) {  // loads first, so their latencies overlap
      const int jj = j + u;
      xj[u] = jj < W ? __ldg(xb + jj) : 1.0f;  // the augmented input's last entry is 1
      if (jj < W && jj < j1) {
        tc[u][0] = p.tr[5][cbase + (long long)jj * M];
        tc[u][1] = p.tr[6][cbase + (long long)jj * M];
      }
      if (jj < j1) {
        tc[u][2] = p.tr[7][kbase + (long long)jj * M];
        tc[u][3] = p.tr[8][kbase + (long long)jj * M];
      }
    }
#pragma unroll
    for (int u = 0; u < kRtrlUnroll; ++u) {
      const int jj = j + u;
      if (jj < W && jj < j1) {
        p.ntr[5][cbase + (long long)jj * M] = adv(tc[u][0], make_float2(k.gsr * xj[u], 0.0f));
        p.ntr[6][cbase + (long long)jj * M] = adv(tc[u][1], make_float2(0.0f, k.gsi * xj[u]));
      }
      if (jj < j1) {
        p.ntr[7][kbase + (long long)jj * M] = adv(tc[u][2], make_float2(xj[u] * k.dph.x, xj[u] * k.dph.y));
        p.ntr[8][kbase + (long long)jj * M] = adv(tc[u][3], make_float2(xj[u] * k.dret.x, xj[u] * k.dret.y));
      }
    }
  }
}

struct RtrlGradParams {
  const float2* g;       // [B, M] (dL/dRe h', dL/dIm h')
  const float2* tr[9];
  const float4* saved;   // [B, M, 2]
  float* grad[9];
  float2* grad_u;        // [B, M] pairs written as [B, 2M] (real half, imaginary half)
  float2* grad_proj;     // [B]
  long long B;
  int W, M, mblocks;
};

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < kRtrlGradThreads / 32; ++w) t += red[w];
  return t;
}

// grid (W + 1 + B + mblocks), 256 threads: CTA j < W + 1 reduces trace row j over the batch
// (content gradients of row j for every mode; for the controllers also over the modes); the
// next B CTAs one batch row each (the content input's gradient and the projections'); the last
// mblocks CTAs 256 modes each (modal gradients). Every sum runs in a fixed order.
__global__ void __launch_bounds__(kRtrlGradThreads) rtrl_grad_kernel(const __grid_constant__ RtrlGradParams p) {
  pdl_wait();
  __shared__ float red[kRtrlGradThreads / 32];
  const int W = p.W, M = p.M;
  const long long B = p.B;
  const int tid = threadIdx.x;
  const long long role = blockIdx.x;
  if (role <= W) {
    const int j = (int)role;
    float sph = 0.0f, sret = 0.0f;
    for (int m = tid; m < M; m += kRtrlGradThreads) {
      // kRtrlUnroll batch rows at a time, their loads issued together; one partial sum per
      // unrolled slot, combined in a fixed order
      float cr[kRtrlUnroll] = {}, ci[kRtrlUnroll] = {}, sp[kRtrlUnroll] = {}, sr[kRtrlUnroll] = {};
      for (long long b0 = 0; b0 < B; b0 += kRtrlUnroll) {
        float2 g[kRtrlUnroll], t[kRtrlUnroll][4];
#pragma unroll
        for (int u = 0; u < kRtrlUnroll; ++u) {
          const long long b = b0 + u;
          if (b < B) {
            g[u] = p.g[b * M + m];
            if (j < W) {
              const long long ci_ = (b * W + j) * (long long)M + m;
              t[u][0] = p.tr[5][ci_];
              t[u][1] = p.tr[6][ci_];
            }
            const long long ki = (b * (W + 1) + j) * (long long)M + m;
            t[u][2] = p.tr[7][ki];
            t[u][3] = p.tr[8][ki];
          }
        }
#pragma unroll
        for (int u = 0; u < kRtrlUnroll; ++u) {
          if (b0 + u < B) {
            if (j < W) {
              cr[u] = fmaf(g[u].x, t[u][0].x, fmaf(g[u].y, t[u][0].y, cr[u]));
              ci[u] = fmaf(g[u].x, t[u][1].x, fmaf(g[u].y, t[u][1].y, ci[u]));
            }
            sp[u] = fmaf(g[u].x, t[u][2].x, fmaf(g[u].y, t[u][2].y, sp[u]));
            sr[u] = fmaf(g[u].x, t[u][3].x, fmaf(g[u].y, t[u][3].y, sr[u]));
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kRtrlUnroll; ++u) {
        sph += sp[u];
        sret += sr[u];
      }
      if (j < W) {
        p.grad[5][(long long)j * M + m] = (cr[0] + cr[1]) + (cr[2] + cr[3]);
        p.grad[6][(long long)j * M + m] = (ci[0] + ci[1]) + (ci[2] + ci[3]);
      }
    }
    sph = block_sum(sph, red);
    sret = block_sum(sret, red);
    if (tid == 0) {
      p.grad[7][j] = sph;
      p.grad[8][j] = sret;
    }
    return;
  }
  if (role <= W + B) {
    const long long b = role - W - 1;
    float s0 = 0.0f, s1 = 0.0f;
    for (int m = tid; m < M; m += kRtrlGradThreads) {
      const float2 g = p.g[b * M + m];
      const float4 v0 = p.saved[(b * M + m) * 2], v1 = p.saved[(b * M + m) * 2 + 1];
      float* gu = reinterpret_cast<float*>(p.grad_u) + b * 2 * M;
      gu[m] = g.x * v0.x;       // dL/du_r = g_r gain slope_r
      gu[M + m] = g.y * v0.y;   // dL/du_i = g_i gain slope_i (u_i writes the imaginary part)
      s0 = fmaf(g.x, v0.z, fmaf(g.y, v0.w, s0));
      s1 = fmaf(g.x, v1.x, fmaf(g.y, v1.y, s1));
    }
    s0 = block_sum(s0, red);
    s1 = block_sum(s1, red);
    if (tid == 0) p.grad_proj[b] = make_float2(s0, s1);
    return;
  }
  const int m = (int)(role - W - 1 - B) * kRtrlGradThreads + tid;
  if (m >= M) return;
  float acc[5] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
  for (long long b = 0; b < B; ++b) {
    const float2 g = p.g[b * M + m];
#pragma unroll
    for (int q = 0; q < 5; ++q) {
      const float2 t = p.tr[q][b * M + m];
      acc[q] = fmaf(g.x, t.x, fmaf(g.y, t.y, acc[q]));
    }
  }
#pragma unroll
  for (int q = 0; q < 5; ++q) p.grad[q][m] = acc[q];
}

static thread_local char g_rtrl_err[256];

static int rtrl_fail(int code, const char* msg) {
  snprintf(g_rtrl_err, sizeof(g_rtrl_err), "%s", msg);
  return code;
}

template <typename P>
static cudaError_t launch_pdl(const void* kernel, dim3 grid, int threads, cudaStream_t s, const P& params) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {const_cast<P*>(&params)};
  return cudaLaunchKernelExC(&cfg, kernel, args);
}

static int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      n = 148;
    }
  }
  return n;
}

}  // namespace sparc

using namespace sparc;

extern "C" {

const char* sparc_rtrl_last_error(void) { return g_rtrl_err; }

int sparc_rtrl_saved_floats(void) { return kRtrlSavedFloats; }

int sparc_rtrl_step(const SparcRtrlStepArgs* a, void* stream) {
  NvtxRange nvtx(__func__);
  if (a == nullptr) return rtrl_fail(SPARC_ERR_ARG, "null args");
  if (a->batch <= 0 || a->input_size <= 0 || a->modes <= 0 || a->batch > 65535)
    return rtrl_fail(SPARC_ERR_SHAPE, "batch (1..65535), input_size and modes must be positive");
  if (!a->x || !a->content || !a->projections || !a->state || !a->new_state || !a->saved || !a->decay_log ||
      !a->frequency_log || !a->write_log_gain || !a->write_phase_response || !a->write_retention_response)
    return rtrl_fail(SPARC_ERR_ARG, "null tensor pointer");
  RtrlStepParams p;
  for (int q = 0; q < 9; ++q) {
    if (!a->traces[q] || !a->new_traces[q]) return rtrl_fail(SPARC_ERR_ARG, "null trace pointer");
    p.tr[q] = reinterpret_cast<const float2*>(a->traces[q]);
    p.ntr[q] = reinterpret_cast<float2*>(a->new_traces[q]);
  }
  p.x = a->x;
  p.u = a->content;
  p.proj = reinterpret_cast<const float2*>(a->projections);
  p.reset = a->reset;
  p.state = reinterpret_cast<const float2*>(a->state);
  p.new_state = reinterpret_cast<float2*>(a->new_state);
  p.dlog = a->decay_log;
  p.flog = a->frequency_log;
  p.wlg = a->write_log_gain;
  p.wpr = a->write_phase_response;
  p.wrr = a->write_retention_response;
  p.saved = reinterpret_cast<float4*>(a->saved);
  p.B = a->batch;
  p.W = a->input_size;
  p.M = a->modes;
  p.lin = a->content_linear ? 1 : 0;
  // split the W + 1 trace rows so that the grid covers the GPU about four times over, with at
  // least eight rows per thread
  const int mblocks = (a->modes + kRtrlThreads - 1) / kRtrlThreads;
  const long long base = (long long)mblocks * a->batch;
  const int rows = a->input_size + 1;
  long long z = std::max<long long>(1, (4LL * sm_count() + base - 1) / base);
  z = std::min<long long>(z, std::max(1, rows / 8));
  z = std::min<long long>(z, 65535);
  p.rows_per_z = (rows + (int)z - 1) / (int)z;
  const int nz = (rows + p.rows_per_z - 1) / p.rows_per_z;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  TimedLaunch tl(kTimeRtrlStep, s);
  const cudaError_t e = launch_pdl((const void*)rtrl_step_kernel, dim3(mblocks, (unsigned)a->batch, nz), kRtrlThreads, s, p);
  return e == cudaSuccess ? SPARC_OK : rtrl_fail(SPARC_ERR_LAUNCH, cudaGetErrorString(e));
}

int sparc_rtrl_grad(const SparcRtrlGradArgs* a, void* stream) {
  NvtxRange nvtx(__func__);
  if (a == nullptr) return rtrl_fail(SPARC_ERR_ARG, "null args");
  if (a->batch <= 0 || a->input_size <= 0 || a->modes <= 0)
    return rtrl_fail(SPARC_ERR_SHAPE, "batch, input_size and modes must be positive");
  if (!a->grad_state || !a->saved || !a->grad_content || !a->grad_projections)
    return rtrl_fail(SPARC_ERR_ARG, "null tensor pointer");
  RtrlGradParams p;
  for (int q = 0; q < 9; ++q) {
    if (!a->traces[q] || !a->grad_params[q]) return rtrl_fail(SPARC_ERR_ARG, "null trace / gradient pointer");
    p.tr[q] = reinterpret_cast<const float2*>(a->traces[q]);
    p.grad[q] = a->grad_params[q];
  }
  p.g = reinterpret_cast<const float2*>(a->grad_state);
  p.saved = reinterpret_cast<const float4*>(a->saved);
  p.grad_u = reinterpret_cast<float2*>(a->grad_content);
  p.grad_proj = reinterpret_cast<float2*>(a->grad_projections);
  p.B = a->batch;
  p.W = a->input_size;
  p.M = a->modes;
  p.mblocks = (a->modes + kRtrlGradThreads - 1) / kRtrlGradThreads;
  const long long grid = (long long)a->input_size + 1 + a->batch + p.mblocks;
  if (grid >= (1LL << 31)) return rtrl_fail(SPARC_ERR_SHAPE, "too many trace rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  TimedLaunch tl(kTimeRtrlGrad, s);
  const cudaError_t e = launch_pdl((const void*)rtrl_grad_kernel, dim3((unsigned)grid), kRtrlGradThreads, s, p);
  return e == cudaSuccess ? SPARC_OK : rtrl_fail(SPARC_ERR_LAUNCH, cudaGetErrorString(e));
}

}  // extern "C"
