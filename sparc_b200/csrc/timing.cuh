// Per-kernel device-time diagnostics shared by the launch sites (definitions in timing.cu), and
// the NVTX range every C-ABI compute entry point opens for its call.
#pragma once

#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

namespace sparc {

// An NVTX range named after the entry point, open for the whole call (validation and launches):
// `ncu --nvtx --nvtx-include "sparc_mixer_backward/"` selects that call's kernels, nsys shows the
// calls on the host timeline. Header-only NVTX v3: without a tool attached a push/pop is a call
// through a no-op function pointer.
class NvtxRange {
 public:
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

enum KernelId {
  kTimeFwdSummary = 0,
  kTimeFwdScan,
  kTimeFwdReplay,
  kTimeBwdSummary,
  kTimeBwdScan,
  kTimeBwdGrad,
  kTimeBwdReduce,
  kTimeRealFwd,
  kTimeRealBwd,
  kTimeDecode,
  kTimeRtrlStep,
  kTimeRtrlGrad,
  kTimeProjGemm,
  kTimePeerAllreduce,
  kTimeProjRowdot,
  kTimeProjColsum,
  kTimeProjGemmFinish,
  kTimeComplexFwdSummary,
  kTimeComplexFwdScan,
  kTimeComplexFwdReplay,
  kTimeComplexBwdSummary,
  kTimeComplexBwdScan,
  kTimeComplexBwdGrad,
  kTimeKernels
};

// While timing is enabled (sparc_timing_enable), brackets one launch with CUDA events on its
// stream; otherwise (or while the stream is being captured) does nothing.
class TimedLaunch {
 public:
  TimedLaunch(int id, cudaStream_t s);
  ~TimedLaunch();
  TimedLaunch(const TimedLaunch&) = delete;
  TimedLaunch& operator=(const TimedLaunch&) = delete;

 private:
  int id_;
  cudaStream_t s_;
  cudaEvent_t start_ = nullptr;
  cudaEvent_t end_ = nullptr;
};

}  // namespace sparc
