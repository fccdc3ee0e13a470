// Shared device helpers for the SPARC B200 kernels (sm_100a).
//
// * Activation I/O types (float / bfloat16) converted to float in registers.
// * Transcendentals. The hardware approximations (ex2/rcp/sqrt/tanh .approx PTX
//   instructions, documented in the PTX ISA) are used directly; the two functions that need
//   more care are built here from textbook series:
//     - tanh for |x| < 1/2 from its Maclaurin series (coefficients from the Bernoulli
//       numbers, 2^{2n}(2^{2n}-1)B_{2n}/(2n)!), else 1 - 2/(e^{2|x|}+1);
//     - -expm1(-u) for u < 1/4 from its Maclaurin series u - u^2/2 + u^3/6 - ...;
//     - sin/cos on [-pi/2, pi/2] from their Maclaurin series (no range reduction needed:
//       the per-token phase offset (1-rho)*delta is bounded by pi/2 in magnitude).
// * Decoupled-lookback flags: a 32-bit word = (epoch << 2) | state. The epoch is bumped by
//   the last CTA of every launch, so flags never need clearing between launches. Every wait
//   is bounded; on timeout the kernel records an error bit in the launch status word and
//   continues with a zero carry, so the launch still terminates.
// * Packed f32x2 arithmetic (add/sub/mul/fma.rn.f32x2) and complex pairs on it.
// * mbarrier, TMA tensor-map and 1-D bulk-copy wrappers (no multicast), programmatic dependent
//   launch.
// * warp_exchange: one warp's values summed over the ranks of a data-parallel group through
//   NVLink peer memory (bounded waits).
// * fail(): the host-side error report of the mixer, decode and real-scan entry points.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sparc {

// Host: records `msg` as the thread-local message sparc_last_error() returns and returns
// `code` (defined in mixer.cu).
int fail(int code, const char* msg);

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn16 = 2.772588722239781f;
constexpr float kHalfPi = 1.5707963267948966f;
constexpr float kInvLn16 = 0.36067376022224085f;   // 1 / ln 16
constexpr float kInvHalfPi = 0.6366197723675814f;  // 2 / pi

// ---------------------------------------------------------------- I/O types
template <typename T> struct Io;
template <> struct Io<float> {
  static __device__ __forceinline__ float load(const float* p) { return __ldg(p); }
  static __device__ __forceinline__ void store(float* p, float v) { *p = v; }
};
template <> struct Io<__nv_bfloat16> {
  static __device__ __forceinline__ float load(const __nv_bfloat16* p) {
    return __bfloat162float(__ldg(p));
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float v) {
    *p = __float2bfloat16_rn(v);
  }
};

__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }

// ---------------------------------------------------------------- math
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float sqrt_approx(float x) {
  float y;
  asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float tanh_hw(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// sin / cos by the hardware approximations (sin.approx / cos.approx, absolute error about 1e-6
// for the arguments used here): the bfloat16 path's transitions.
__device__ __forceinline__ void sincos_hw(float x, float* s, float* c) {
  asm("sin.approx.ftz.f32 %0, %1;" : "=f"(*s) : "f"(x));
  asm("cos.approx.ftz.f32 %0, %1;" : "=f"(*c) : "f"(x));
}

// tanh accurate to a few float32 ulp: Maclaurin series below 1/2, exponential form above.
__device__ __forceinline__ float tanh_accurate(float x) {
  const float ax = fabsf(x);
  const float e = ex2_approx(2.0f * kLog2e * ax);
  const float big = 1.0f - 2.0f * rcp_approx(e + 1.0f);
  const float x2 = x * x;
  // 1, -1/3, 2/15, -17/315, 62/2835, -1382/155925, 21844/6081075, -929569/638512875
  float p = -1.4558343870513183e-3f;
  p = fmaf(p, x2, 3.5921280365724810e-3f);
  p = fmaf(p, x2, -8.8632355299021966e-3f);
  p = fmaf(p, x2, 2.1869488536155203e-2f);
  p = fmaf(p, x2, -5.3968253968253968e-2f);
  p = fmaf(p, x2, 1.3333333333333333e-1f);
  p = fmaf(p, x2, -3.3333333333333333e-1f);
  const float small = fmaf(p * x2, x, x);
  return ax < 0.5f ? small : copysignf(big, x);
}

// sin and cos of |x| <= pi/2 (Maclaurin series through x^13 / x^12).
__device__ __forceinline__ void sincos_halfpi(float x, float* s, float* c) {
  const float x2 = x * x;
  float ps = 1.6059043836821615e-10f;         // 1/13!
  ps = fmaf(ps, x2, -2.5052108385441720e-8f);  // -1/11!
  ps = fmaf(ps, x2, 2.7557319223985893e-6f);   // 1/9!
  ps = fmaf(ps, x2, -1.9841269841269841e-4f);  // -1/7!
  ps = fmaf(ps, x2, 8.3333333333333333e-3f);   // 1/5!
  ps = fmaf(ps, x2, -1.6666666666666667e-1f);  // -1/3!
  *s = fmaf(ps * x2, x, x);
  float pc = 2.0876756987868099e-9f;           // 1/12!
  pc = fmaf(pc, x2, -2.7557319223985891e-7f);  // -1/10!
  pc = fmaf(pc, x2, 2.4801587301587302e-5f);   // 1/8!
  pc = fmaf(pc, x2, -1.3888888888888889e-3f);  // -1/6!
  pc = fmaf(pc, x2, 4.1666666666666667e-2f);   // 1/4!
  pc = fmaf(pc, x2, -0.5f);
  *c = fmaf(pc, x2, 1.0f);
}

// ---------------------------------------------------------------- launch state + lookback
struct LaunchState {
  unsigned epoch;   // bumped by the last CTA of each launch
  unsigned ticket;  // dynamic tile counter, reset by the last CTA
  unsigned done;    // CTAs finished in this launch
  unsigned status;  // sticky error bits (kStatusTimeout ...)
  unsigned pad[60];
};
static_assert(sizeof(LaunchState) == 256, "launch state is one 256-byte line");

constexpr unsigned kStatusTimeout = 1u;
constexpr unsigned kFlagAggregate = 1u;
constexpr unsigned kFlagInclusive = 2u;

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Spin (bounded) until the flag carries this epoch and a state >= min_state. Returns the
// state, or 0 after `max_spin` polls (the caller then records a timeout).
__device__ __forceinline__ unsigned wait_flag(const unsigned* flag, unsigned epoch,
                                              unsigned max_spin, unsigned min_state = 1u) {
  for (unsigned it = 0; it < max_spin; ++it) {
    const unsigned v = ld_acquire(flag);
    if ((v >> 2) == (epoch & 0x3fffffffu) && (v & 3u) >= min_state) return v & 3u;
    if (it > 8) __nanosleep(it < 64 ? 32 : 256);
  }
  return 0u;
}

__device__ __forceinline__ unsigned make_flag(unsigned epoch, unsigned state) {
  return ((epoch & 0x3fffffffu) << 2) | state;
}

// Called once per CTA at the very end of a persistent kernel: the last CTA resets the ticket
// and bumps the epoch so the next launch on this workspace starts clean.
__device__ __forceinline__ void finish_launch(LaunchState* ls) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned total = gridDim.x * gridDim.y * gridDim.z;
    const unsigned prev = atomicAdd(&ls->done, 1u);
    if (prev == total - 1u) {
      ls->ticket = 0u;
      ls->done = 0u;
      __threadfence();
      atomicAdd(&ls->epoch, 1u);
    }
  }
}

// ---------------------------------------------------------------- packed float pairs
// sm_100's f32x2 arithmetic applies one add / sub / mul / fma to both lanes of a register pair
// in one instruction (here the lanes are the two modes a thread owns). The .rn forms round like
// the scalar operations.
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
  float2 d;
  asm("{.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "sub.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {  // a*b + c
  float2 d;
  asm("{.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 bcast2(float v) { return make_float2(v, v); }

// Two modes' complex numbers: re = (re0, re1), im = (im0, im1).
struct Cx2 {
  float2 re, im;
};
__device__ __forceinline__ Cx2 cx2(float2 re, float2 im) { return Cx2{re, im}; }
__device__ __forceinline__ Cx2 cmul2(Cx2 a, Cx2 b) {
  return Cx2{sub2(mul2(a.re, b.re), mul2(a.im, b.im)), fma2(a.re, b.im, mul2(a.im, b.re))};
}
__device__ __forceinline__ Cx2 cfma2(Cx2 a, Cx2 b, Cx2 c) {  // a*b + c
  return Cx2{sub2(fma2(a.re, b.re, c.re), mul2(a.im, b.im)), fma2(a.re, b.im, fma2(a.im, b.re, c.im))};
}

// Per-lane hardware approximations on pairs.
__device__ __forceinline__ float2 ex2_2(float2 v) { return make_float2(ex2_approx(v.x), ex2_approx(v.y)); }
__device__ __forceinline__ float2 rcp_2(float2 v) { return make_float2(rcp_approx(v.x), rcp_approx(v.y)); }
__device__ __forceinline__ float2 sqrt_2(float2 v) { return make_float2(sqrt_approx(v.x), sqrt_approx(v.y)); }
__device__ __forceinline__ float2 tanh_hw2(float2 v) { return make_float2(tanh_hw(v.x), tanh_hw(v.y)); }

// tanh of a pair (the float32 content of every (token, mode)): 1 - 2 / (e^{2x} + 1) with the
// hardware exp2 and reciprocal approximations. Its absolute error is a few units of 2^-24 for
// every x (x -> +inf gives 1, x -> -inf gives -1); only where |tanh x| is itself that small is
// the relative error large, which the float32 tolerances (relative l2 norms over whole tensors)
// do not see.
__device__ __forceinline__ float2 tanh_exp2(float2 x) {
  const float2 e = ex2_2(mul2(bcast2(2.0f * kLog2e), x));
  const float2 r = rcp_2(add2(e, bcast2(1.0f)));
  return fma2(bcast2(-2.0f), r, bcast2(1.0f));
}
template <bool kFast>
__device__ __forceinline__ float2 tanh_t2(float2 x) {
  if constexpr (kFast) return tanh_hw2(x);
  else return tanh_exp2(x);
}

// Packed forms of the series helpers above (same coefficients and branch points, per lane).
// -expm1(-u) = 1 - e^{-u} for u >= 0, given w = e^{-u}, per lane: the series
// u - u^2/2 + u^3/6 - u^4/24 + u^5/120 - u^6/720 below 1/4 (cancellation-free), else 1 - w.
__device__ __forceinline__ float2 one_minus_exp_neg2(float2 u, float2 w) {
  float2 p = bcast2(-1.3888888888888889e-3f);
  p = fma2(p, u, bcast2(8.3333333333333333e-3f));
  p = fma2(p, u, bcast2(-4.1666666666666667e-2f));
  p = fma2(p, u, bcast2(1.6666666666666667e-1f));
  p = fma2(p, u, bcast2(-0.5f));
  p = fma2(p, u, bcast2(1.0f));
  const float2 small = mul2(p, u);
  const float2 big = sub2(bcast2(1.0f), w);
  return make_float2(u.x < 0.25f ? small.x : big.x, u.y < 0.25f ? small.y : big.y);
}
__device__ __forceinline__ void sincos_halfpi2(float2 x, float2* s, float2* c) {
  const float2 x2 = mul2(x, x);
  float2 ps = bcast2(1.6059043836821615e-10f);
  ps = fma2(ps, x2, bcast2(-2.5052108385441720e-8f));
  ps = fma2(ps, x2, bcast2(2.7557319223985893e-6f));
  ps = fma2(ps, x2, bcast2(-1.9841269841269841e-4f));
  ps = fma2(ps, x2, bcast2(8.3333333333333333e-3f));
  ps = fma2(ps, x2, bcast2(-1.6666666666666667e-1f));
  *s = fma2(mul2(ps, x2), x, x);
  float2 pc = bcast2(2.0876756987868099e-9f);
  pc = fma2(pc, x2, bcast2(-2.7557319223985891e-7f));
  pc = fma2(pc, x2, bcast2(2.4801587301587302e-5f));
  pc = fma2(pc, x2, bcast2(-1.3888888888888889e-3f));
  pc = fma2(pc, x2, bcast2(4.1666666666666667e-2f));
  pc = fma2(pc, x2, bcast2(-0.5f));
  *c = fma2(pc, x2, bcast2(1.0f));
}

// Programmatic dependent launch: kernels are launched so that they may start while the previous
// kernel on the stream drains; this waits until that kernel has completed and its memory is
// visible (a no-op when the launch had no programmatic dependency). Nothing the previous kernel
// writes may be read before it. Kernels here do not trigger their dependents early (measured
// slower at the config-5 sizes), so a launch starts once every CTA of the previous kernel has
// exited, each after its own wait: the kernels before the previous one have then completed, and
// their outputs may be read (prefetched) before this wait.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Complex helpers on float2 (x = real, y = imag).
__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(fmaf(a.x, b.x, -a.y * b.y), fmaf(a.x, b.y, a.y * b.x));
}
__device__ __forceinline__ float2 cfma(float2 a, float2 b, float2 c) {  // a*b + c
  return make_float2(fmaf(a.x, b.x, fmaf(-a.y, b.y, c.x)), fmaf(a.x, b.y, fmaf(a.y, b.x, c.y)));
}

}  // namespace sparc

namespace sparc {

// ---------------------------------------------------------------- TMA bulk copies + mbarriers
// 1-D bulk copies (cp.async.bulk, no tensor map, no multicast) from global into this CTA's
// shared memory, completing on an mbarrier with a transaction count. Source and destination
// must be 16-byte aligned and the size a multiple of 16.
__device__ __forceinline__ unsigned smem_addr(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned long long* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0u;
}
// Bounded wait for the phase with the given parity; false after max_spin polls.
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, unsigned parity, unsigned max_spin) {
  for (unsigned it = 0; it < max_spin; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  return false;
}
// Bounded wait that also acquires at cluster scope: for data that other CTAs of the cluster
// stored into this CTA's shared memory with st_async_f32 (completing on this barrier).
__device__ __forceinline__ bool mbar_wait_cluster(unsigned long long* bar, unsigned parity, unsigned max_spin) {
  for (unsigned it = 0; it < max_spin; ++it) {
    unsigned ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}
// The shared::cluster address of this CTA's shared-memory object `p` in cluster CTA `rank`.
__device__ __forceinline__ unsigned cluster_smem_addr(const void* p, unsigned rank) {
  unsigned r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
  return r;
}
// Asynchronous 4-byte store into a cluster CTA's shared memory that completes 4 bytes of the
// transaction count of that CTA's mbarrier (both addresses from cluster_smem_addr): no fence
// or cluster barrier is needed, the receiver's wait on its barrier sees the data.
__device__ __forceinline__ void st_async_f32(unsigned raddr, float v, unsigned rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(raddr), "f"(v),
               "r"(rbar)
               : "memory");
}
// A cluster barrier for CTA lifetime only (no CTA leaves while a peer may still access its
// shared memory), with no memory ordering: the peers' accesses before it have completed (their
// values were used before the arrive issued), and nothing written before it needs to be seen by a
// peer, so the arrive does not wait for this CTA's outstanding global stores as the ordered
// (release) form does.
__device__ __forceinline__ void cluster_sync_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, unsigned bytes,
                                              unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// TMA tile load of a 3-D box described by a tensor map (no multicast) into this CTA's shared
// memory, completing on an mbarrier. The map must live in kernel-parameter space
// (__grid_constant__); c0 is the innermost coordinate (its byte offset must be 16-aligned).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<unsigned long long>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
      : "memory");
}

// ---------------------------------------------------------------- peer exchange (N GPUs)
// One warp's values summed over the ranks of a data-parallel group through NVLink peer memory,
// inside the kernel that computed them (the parameter-gradient reduction). Every rank holds an
// exchange buffer mapped into every rank (CUDA IPC):
//   epoch [kXchgSlots] u32, inbox [2][world][kXchgSlots][32] u64.
// A slot is one warp-sized group of values of one launch geometry; its epoch counts the
// launches that used it. Each lane stores its value together with the epoch e as one 8-byte word
// (value in the low half, e in the high half: a naturally aligned 8-byte store is single-copy
// atomic, so a reader that sees e sees the value stored with it) into inbox[e & 1][rank][slot]
// of every rank, then waits (bounded) until the word from every rank carries e in its own inbox,
// and sums the ranks' values in rank order: every rank gets the identical sum. No fence and no
// separate flag: one NVLink write per value is the whole exchange. A peer can run one exchange
// ahead on a slot (the parity double-buffers the inbox) but not two (it needs this rank's next
// push first), so a word of the other parity is never overwritten while it is awaited.
constexpr int kXchgSlots = 1024;
constexpr int kXchgMaxRanks = 8;
constexpr unsigned kStatusXchgTimeout = 16u;

struct PeerExchange {
  unsigned char* base[kXchgMaxRanks];  // every rank's exchange buffer, as mapped here
  int world, rank;                     // world <= 1: no exchange
  unsigned* status;
  unsigned max_spin;
};

__host__ __device__ constexpr size_t xchg_inbox_offset() { return (size_t)kXchgSlots * 4; }
__host__ __device__ constexpr size_t xchg_buffer_bytes(int world) {
  return xchg_inbox_offset() + 2 * (size_t)world * kXchgSlots * 32 * 8;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Called by all 32 lanes of one warp with the lane's value; returns the sum over the ranks.
__device__ __forceinline__ float warp_exchange(const PeerExchange& x, int slot, float val) {
  const int lane = threadIdx.x & 31;
  unsigned* epoch = reinterpret_cast<unsigned*>(x.base[x.rank]) + slot;
  unsigned e = 0;
  if (lane == 0) e = *epoch + 1u;
  e = __shfl_sync(0xffffffffu, e, 0);
  const long long par = e & 1u;
  const unsigned long long word = ((unsigned long long)e << 32) | (unsigned long long)__float_as_uint(val);
  for (int r = 0; r < x.world; ++r) {
    unsigned long long* in = reinterpret_cast<unsigned long long*>(x.base[r] + xchg_inbox_offset());
    st_relaxed_sys_u64(in + ((par * x.world + x.rank) * kXchgSlots + slot) * 32 + lane, word);
  }
  const unsigned long long* own = reinterpret_cast<const unsigned long long*>(x.base[x.rank] + xchg_inbox_offset());
  float v[kXchgMaxRanks];
  bool late = false;
#pragma unroll
  for (int r = 0; r < kXchgMaxRanks; ++r) {
    v[r] = 0.0f;
    if (r < x.world) {
      const unsigned long long* w = own + ((par * x.world + r) * kXchgSlots + slot) * 32 + lane;
      unsigned long long got = ld_relaxed_sys_u64(w);
      unsigned it = 0;
      while ((unsigned)(got >> 32) != e) {
        if (++it >= x.max_spin) {
          late = true;
          break;
        }
        __nanosleep(32);
        got = ld_relaxed_sys_u64(w);
      }
      v[r] = __uint_as_float((unsigned)got);
    }
  }
  if (late) atomicOr(x.status, kStatusXchgTimeout);
  float s = 0.0f;
#pragma unroll
  for (int r = 0; r < kXchgMaxRanks; ++r)
    if (r < x.world) s += v[r];
  __syncwarp();
  if (lane == 0) *epoch = e;
  return s;
}

}  // namespace sparc

