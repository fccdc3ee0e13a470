// Generic complex diagonal scan h_t = a_t h_{t-1} + b_t (h_{-1} = 0) for B200 (sm_100a), forward
// and backward: the reference's complex_scan / complex_scan_with_last (backward/scan.py:887-919,
// 1653-1656, 1838-1855; kernels forward/scan.py:701-722 and backward/scan.py:131-160).
//
// Parity rules kept from the reference: every operand is read in its own dtype and widened to
// float32 (here: ar/ai in one dtype, br/bi in another); the outputs have b's dtype, the last
// state is float32; the backward reads the forward's outputs (b's dtype) as the previous states,
// accumulates the adjoint adj_t = grad_t + conj(a_{t+1}) adj_{t+1} in float32, and writes all
// four gradients in a's dtype:
//   grad_ar = Re(adj) Re(h_{t-1}) + Im(adj) Im(h_{t-1}),
//   grad_ai = Im(adj) Re(h_{t-1}) - Re(adj) Im(h_{t-1}),  grad_b = adj.
//
// Decomposition (three launches each way, no waits between CTAs): the sequence is cut into
// chunks of kCxChunk tokens. A summary kernel composes each chunk's affine map h_out = P h_in + Q
// (forward) or adj_out = R adj_in + S (backward, conj(a) multipliers, tokens in reverse) per
// (batch row, chunk, mode); the mixer's cluster carry scan (launch_chunk_carry_scan, mixer.cu)
// turns the maps into the value leaving every chunk; a replay kernel runs the recurrence through
// each chunk from its carried-in value, writing the outputs and the last state (forward) or the
// gradients (backward). Thread per mode, 128 modes per CTA, one CTA per (mode block, chunk, batch row);
// each thread issues a group of kCxUnroll tokens' loads before using them (the replay kernel is
// held to six CTAs' worth of registers: left alone it takes 143 and three CTAs per SM, too few
// loads in flight).
#include <algorithm>

#include "common.cuh"
#include "sparc_b200.h"
#include "timing.cuh"

namespace sparc {

constexpr int kCxChunk = 32;    // tokens per chunk map
constexpr int kCxModes = 128;   // modes (threads) per CTA
constexpr int kCxUnroll = 8;    // tokens whose loads are issued together

// The mixer's chunk carry scan over maps [rows, chunks, M] float4 (A.re, A.im, B.re, B.im):
// out[r, c] = the value after chunk c (forward order, or from the last chunk backwards with
// `reverse`), starting from zero; final_r/final_i (optional) receive the value after the last
// chunk processed. Defined in mixer.cu.
cudaError_t launch_chunk_carry_scan(const float4* maps, float2* out, int rows, int M, int chunks, int reverse,
                                    float* final_r, float* final_i, cudaStream_t s);

struct CxParams {
  const void* ar;
  const void* ai;
  const void* br;
  const void* bi;
  void* out_r;        // forward outputs / the backward's saved outputs (b's dtype)
  void* out_i;
  const void* gr;     // backward: grad of out_r, out_i (b's dtype)
  const void* gi;
  void* gar;          // backward: gradients (a's dtype)
  void* gai;
  void* gbr;
  void* gbi;
  float4* maps;       // [B, chunks, M]
  float2* carry;      // [B, chunks, M]: value leaving each chunk
  float* last_r;      // forward: [B, M] float32 final state, or null
  float* last_i;
  long long L;
  int M, chunks;
};

template <typename T>
__device__ __forceinline__ float ld(const void* p, long long i) {
  return Io<T>::load(static_cast<const T*>(p) + i);
}
template <typename T>
__device__ __forceinline__ void st(void* p, long long i, float v) {
  Io<T>::store(static_cast<T*>(p) + i, v);
}

// Forward chunk map: Q = h after the chunk from h_in = 0, P = product of the a's.
template <typename TA, typename TB>
__global__ void __launch_bounds__(kCxModes) complex_fwd_summary_kernel(const CxParams p) {
  pdl_wait();
  const int m = blockIdx.x * kCxModes + threadIdx.x;
  if (m >= p.M) return;
  const long long t0 = (long long)blockIdx.y * kCxChunk;
  const int n = (int)(p.L - t0 < kCxChunk ? p.L - t0 : kCxChunk);
  const long long base = ((long long)blockIdx.z * p.L + t0) * p.M + m;
  float2 P = make_float2(1.0f, 0.0f), Q = make_float2(0.0f, 0.0f);
  for (int u0 = 0; u0 < n; u0 += kCxUnroll) {
    float2 a[kCxUnroll], b[kCxUnroll];
#pragma unroll
    for (int u = 0; u < kCxUnroll; ++u) {
      const long long i = base + (long long)(u0 + u) * p.M;
      const bool ok = u0 + u < n;
      a[u] = ok ? make_float2(ld<TA>(p.ar, i), ld<TA>(p.ai, i)) : make_float2(1.0f, 0.0f);
      b[u] = ok ? make_float2(ld<TB>(p.br, i), ld<TB>(p.bi, i)) : make_float2(0.0f, 0.0f);
    }
#pragma unroll
    for (int u = 0; u < kCxUnroll; ++u) {
      Q = cfma(a[u], Q, b[u]);
      P = cmul(a[u], P);
    }
  }
  p.maps[((long long)blockIdx.z * p.chunks + blockIdx.y) * p.M + m] = make_float4(P.x, P.y, Q.x, Q.y);
}

// Forward replay: h from the state entering the chunk, outputs in b's dtype.
template <typename TA, typename TB>
__global__ void __launch_bounds__(kCxModes, 6) complex_fwd_replay_kernel(const CxParams p) {
  pdl_wait();
  const int m = blockIdx.x * kCxModes + threadIdx.x;
  if (m >= p.M) return;
  const long long c = blockIdx.y;
  const long long t0 = c * kCxChunk;
  const int n = (int)(p.L - t0 < kCxChunk ? p.L - t0 : kCxChunk);
  const long long base = ((long long)blockIdx.z * p.L + t0) * p.M + m;
  float2 h = c > 0 ? p.carry[((long long)blockIdx.z * p.chunks + c - 1) * p.M + m] : make_float2(0.0f, 0.0f);
  for (int u0 = 0; u0 < n; u0 += kCxUnroll) {
    float2 a[kCxUnroll], b[kCxUnroll];
#pragma unroll
    for (int u = 0; u < kCxUnroll; ++u) {
      const long long i = base + (long long)(u0 + u) * p.M;
      const bool ok = u0 + u < n;
      a[u] = ok ? make_float2(ld<TA>(p.ar, i), ld<TA>(p.ai, i)) : make_float2(1.0f, 0.0f);
      b[u] = ok ? make_float2(ld<TB>(p.br, i), ld<TB>(p.bi, i)) : make_float2(0.0f, 0.0f);
    }
#pragma unroll
    for (int u = 0; u < kCxUnroll; ++u) {
      h = cfma(a[u], h, b[u]);
      if (u0 + u < n) {
        const long long i = base + (long long)(u0 + u) * p.M;
        st<TB>(p.out_r, i, h.x);
        st<TB>(p.out_i, i, h.y);
      }
    }
  }
  if (p.last_r != nullptr && c == p.chunks - 1) {  // the final state, as the last output has it
    p.last_r[(long long)blockIdx.z * p.M + m] = h.x;
    p.last_i[(long long)blockIdx.z * p.M + m] = h.y;
  }
}

// conj(a) z
__device__ __forceinline__ float2 cjmul(float2 a, float2 z) {
  return make_float2(fmaf(a.x, z.x, a.y * z.y), fmaf(a.x, z.y, -a.y * z.x));
}

// Backward chunk map over the chunk's tokens in reverse: the adjoint leaving the chunk toward
// the previous one is R adj_in + S, adj_in the adjoint entering from the next chunk.
template <typename TA, typename TB>
__global__ void __launch_bounds__(kCxModes) complex_bwd_summary_kernel(const CxParams p) {
  pdl_wait();
  const int m = blockIdx.x * kCxModes + threadIdx.x;
  if (m >= p.M) return;
  const long long t0 = (long long)blockIdx.y * kCxChunk;
  const int n = (int)(p.L - t0 < kCxChunk ? p.L - t0 : kCxChunk);
  const long long base = ((long long)blockIdx.z * p.L + t0) * p.M + m;
  float2 R = make_float2(1.0f, 0.0f), S = make_float2(0.0f, 0.0f);
  for (int u0 = n - 1; u0 >= 0; u0 -= kCxUnroll) {  // tokens u0, u0 - 1, ...
    float2 a[kCxUnroll], g[kCxUnroll];
#pragma unroll
    for (int u = 0; u < kCxUnroll; ++u) {
      const long long i = base + (long long)(u0 - u) * p.M;
      const bool ok = u0 - u >= 0;
      a[u] = ok ? make_float2(ld<TA>(p.ar, i), ld<TA>(p.ai, i)) : make_float2(1.0f, 0.0f);
      g[u] = ok ? make_float2(ld<TB>(p.gr, i), ld<TB>(p.gi, i)) : make_float2(0.0f, 0.0f);
    }
#pragma unroll
    for (int u = 0; u < kCxUnroll; ++u) {
      S = cjmul(a[u], make_float2(S.x + g[u].x, S.y + g[u].y));
      R = cjmul(a[u], R);
    }
  }
  p.maps[((long long)blockIdx.z * p.chunks + blockIdx.y) * p.M + m] = make_float4(R.x, R.y, S.x, S.y);
}

// Backward replay: the adjoint through the chunk in reverse from the one entering it, the
// gradients per token against the saved outputs h_{t-1}.
template <typename TA, typename TB>
__global__ void __launch_bounds__(kCxModes) complex_bwd_grad_kernel(const CxParams p) {
  pdl_wait();
  const int m = blockIdx.x * kCxModes + threadIdx.x;
  if (m >= p.M) return;
  const long long c = blockIdx.y;
  const long long t0 = c * kCxChunk;
  const int n = (int)(p.L - t0 < kCxChunk ? p.L - t0 : kCxChunk);
  const long long base = ((long long)blockIdx.z * p.L + t0) * p.M + m;
  float2 adj = c + 1 < p.chunks ? p.carry[((long long)blockIdx.z * p.chunks + c + 1) * p.M + m]
                                : make_float2(0.0f, 0.0f);
  for (int u0 = n - 1; u0 >= 0; u0 -= kCxUnroll) {
    float2 a[kCxUnroll], g[kCxUnroll], hp[kCxUnroll];
#pragma unroll
    for (int u = 0; u < kCxUnroll; ++u) {
      const int k = u0 - u;  // token within the chunk
      const long long i = base + (long long)k * p.M;
      const bool ok = k >= 0;
      a[u] = ok ? make_float2(ld<TA>(p.ar, i), ld<TA>(p.ai, i)) : make_float2(1.0f, 0.0f);
      g[u] = ok ? make_float2(ld<TB>(p.gr, i), ld<TB>(p.gi, i)) : make_float2(0.0f, 0.0f);
      const bool has_prev = ok && t0 + k > 0;
      hp[u] = has_prev ? make_float2(ld<TB>(p.out_r, i - p.M), ld<TB>(p.out_i, i - p.M)) : make_float2(0.0f, 0.0f);
    }
#pragma unroll
    for (int u = 0; u < kCxUnroll; ++u) {
      const int k = u0 - u;
      adj = make_float2(adj.x + g[u].x, adj.y + g[u].y);
      if (k >= 0) {
        const long long i = base + (long long)k * p.M;
        st<TA>(p.gar, i, fmaf(adj.x, hp[u].x, adj.y * hp[u].y));
        st<TA>(p.gai, i, fmaf(adj.y, hp[u].x, -adj.x * hp[u].y));
        st<TA>(p.gbr, i, adj.x);
        st<TA>(p.gbi, i, adj.y);
      }
      adj = cjmul(a[u], adj);
    }
  }
}

static bool cx_valid_dtype(int d) { return d == SPARC_DTYPE_F32 || d == SPARC_DTYPE_BF16; }

static size_t cx_ws_bytes(long long batch, long long length, long long modes) {
  const long long chunks = (length + kCxChunk - 1) / kCxChunk;
  const size_t n = (size_t)batch * (size_t)chunks * (size_t)modes;
  return 256 + n * sizeof(float4) + n * sizeof(float2);
}

static int cx_check_shape(long long batch, long long length, long long modes) {
  if (batch <= 0 || length <= 0 || modes <= 0) return fail(SPARC_ERR_SHAPE, "batch, length and modes must be positive");
  const long long chunks = (length + kCxChunk - 1) / kCxChunk;
  if (batch > 65535 || chunks > 65535 || modes > (1LL << 30) || batch * chunks * modes >= (1LL << 31) ||
      batch * length * modes >= (1LL << 62))
    return fail(SPARC_ERR_SHAPE, "shape beyond the launch grid (batch <= 65535, length <= 2097120, "
                                 "batch x chunks x modes < 2^31)");
  return SPARC_OK;
}

template <typename TA, typename TB>
static cudaError_t cx_launch(const CxParams& p, long long batch, bool backward, cudaStream_t s) {
  const dim3 grid((unsigned)((p.M + kCxModes - 1) / kCxModes), (unsigned)p.chunks, (unsigned)batch);
  {
    TimedLaunch tl(backward ? kTimeComplexBwdSummary : kTimeComplexFwdSummary, s);
    if (backward)
      complex_bwd_summary_kernel<TA, TB><<<grid, kCxModes, 0, s>>>(p);
    else
      complex_fwd_summary_kernel<TA, TB><<<grid, kCxModes, 0, s>>>(p);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  {
    TimedLaunch tl(backward ? kTimeComplexBwdScan : kTimeComplexFwdScan, s);
    const cudaError_t e =
        launch_chunk_carry_scan(p.maps, p.carry, (int)batch, p.M, p.chunks, backward ? 1 : 0, nullptr, nullptr, s);
    if (e != cudaSuccess) return e;
  }
  TimedLaunch tl(backward ? kTimeComplexBwdGrad : kTimeComplexFwdReplay, s);
  if (backward)
    complex_bwd_grad_kernel<TA, TB><<<grid, kCxModes, 0, s>>>(p);
  else
    complex_fwd_replay_kernel<TA, TB><<<grid, kCxModes, 0, s>>>(p);
  return cudaGetLastError();
}

static int cx_dispatch(const CxParams& p, long long batch, int a_dtype, int b_dtype, bool backward, cudaStream_t s) {
  cudaError_t e;
  const bool abf = a_dtype == SPARC_DTYPE_BF16, bbf = b_dtype == SPARC_DTYPE_BF16;
  if (abf && bbf)
    e = cx_launch<__nv_bfloat16, __nv_bfloat16>(p, batch, backward, s);
  else if (abf)
    e = cx_launch<__nv_bfloat16, float>(p, batch, backward, s);
  else if (bbf)
    e = cx_launch<float, __nv_bfloat16>(p, batch, backward, s);
  else
    e = cx_launch<float, float>(p, batch, backward, s);
  if (e != cudaSuccess) return fail(SPARC_ERR_LAUNCH, cudaGetErrorString(e));
  return SPARC_OK;
}

static void cx_workspace(CxParams* p, void* ws, long long batch) {
  const size_t n = (size_t)batch * (size_t)p->chunks * (size_t)p->M;
  char* base = static_cast<char*>(ws) + 256;
  p->maps = reinterpret_cast<float4*>(base);
  p->carry = reinterpret_cast<float2*>(base + n * sizeof(float4));
}

}  // namespace sparc

using namespace sparc;

extern "C" {

long long sparc_complex_chunk_tokens(void) { return kCxChunk; }

size_t sparc_complex_workspace_bytes(long long batch, long long length, long long modes) {
  if (cx_check_shape(batch, length, modes) != SPARC_OK) return 0;
  return cx_ws_bytes(batch, length, modes);
}

int sparc_complex_scan_forward(const SparcComplexFwdArgs* a, void* stream) {
  NvtxRange nvtx(__func__);
  if (a == nullptr) return fail(SPARC_ERR_ARG, "null args");
  if (!a->ar || !a->ai || !a->br || !a->bi || !a->out_r || !a->out_i || !a->workspace)
    return fail(SPARC_ERR_ARG, "null tensor pointer");
  if ((a->last_r == nullptr) != (a->last_i == nullptr)) return fail(SPARC_ERR_ARG, "last_r and last_i go together");
  const int rc = cx_check_shape(a->batch, a->length, a->modes);
  if (rc != SPARC_OK) return rc;
  if (!cx_valid_dtype(a->a_dtype) || !cx_valid_dtype(a->b_dtype)) return fail(SPARC_ERR_DTYPE, "unsupported dtype");
  if (a->workspace_bytes < cx_ws_bytes(a->batch, a->length, a->modes) ||
      reinterpret_cast<uintptr_t>(a->workspace) % 16 != 0)
    return fail(SPARC_ERR_WORKSPACE, "workspace too small or not 16-byte aligned");
  CxParams p = {};
  p.ar = a->ar;
  p.ai = a->ai;
  p.br = a->br;
  p.bi = a->bi;
  p.out_r = a->out_r;
  p.out_i = a->out_i;
  p.L = a->length;
  p.M = (int)a->modes;
  p.chunks = (int)((a->length + kCxChunk - 1) / kCxChunk);
  cx_workspace(&p, a->workspace, a->batch);
  p.last_r = a->last_r;
  p.last_i = a->last_i;
  return cx_dispatch(p, a->batch, a->a_dtype, a->b_dtype, false, static_cast<cudaStream_t>(stream));
}

int sparc_complex_scan_backward(const SparcComplexBwdArgs* a, void* stream) {
  NvtxRange nvtx(__func__);
  if (a == nullptr) return fail(SPARC_ERR_ARG, "null args");
  if (!a->ar || !a->ai || !a->out_r || !a->out_i || !a->grad_out_r || !a->grad_out_i || !a->grad_ar ||
      !a->grad_ai || !a->grad_br || !a->grad_bi || !a->workspace)
    return fail(SPARC_ERR_ARG, "null tensor pointer");
  const int rc = cx_check_shape(a->batch, a->length, a->modes);
  if (rc != SPARC_OK) return rc;
  if (!cx_valid_dtype(a->a_dtype) || !cx_valid_dtype(a->b_dtype)) return fail(SPARC_ERR_DTYPE, "unsupported dtype");
  if (a->workspace_bytes < cx_ws_bytes(a->batch, a->length, a->modes) ||
      reinterpret_cast<uintptr_t>(a->workspace) % 16 != 0)
    return fail(SPARC_ERR_WORKSPACE, "workspace too small or not 16-byte aligned");
  CxParams p = {};
  p.ar = a->ar;
  p.ai = a->ai;
  p.out_r = const_cast<void*>(a->out_r);
  p.out_i = const_cast<void*>(a->out_i);
  p.gr = a->grad_out_r;
  p.gi = a->grad_out_i;
  p.gar = a->grad_ar;
  p.gai = a->grad_ai;
  p.gbr = a->grad_br;
  p.gbi = a->grad_bi;
  p.L = a->length;
  p.M = (int)a->modes;
  p.chunks = (int)((a->length + kCxChunk - 1) / kCxChunk);
  cx_workspace(&p, a->workspace, a->batch);
  return cx_dispatch(p, a->batch, a->a_dtype, a->b_dtype, true, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
