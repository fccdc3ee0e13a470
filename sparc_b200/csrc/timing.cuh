// Per-kernel device-time diagnostics shared by the launch sites (definitions in timing.cu).
#pragma once

#include <cuda_runtime.h>

namespace sparc {

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
