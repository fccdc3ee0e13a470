// Per-kernel device-time diagnostics: CUDA events around each launch while enabled, collected
// and summed per kernel kind by sparc_timing_read. Events come from a small pool so that a
// timing loop does not create and destroy events per launch.
#include <atomic>
#include <mutex>
#include <vector>

#include "sparc_b200.h"
#include "timing.cuh"

namespace sparc {
namespace {

struct Pending {
  int id;
  cudaEvent_t start, end;
};

std::atomic<int> g_on{0};
std::mutex g_mu;
std::vector<cudaEvent_t> g_pool;
std::vector<Pending> g_pending;
double g_ms[kTimeKernels] = {};
long long g_count[kTimeKernels] = {};

const char* const kNames[kTimeKernels] = {
    "mixer_fwd_summary_kernel", "mixer_carry_scan_kernel(fwd)", "mixer_fwd_replay_kernel",
    "mixer_bwd_summary_kernel", "mixer_carry_scan_kernel(bwd)", "mixer_bwd_grad_kernel",
    "mixer_reduce_kernel",      "real_fwd_kernel",              "real_bwd_kernel",
    "decode_kernel",            "rtrl_step_kernel",             "rtrl_grad_kernel",
    "proj_gemm_kernel",         "peer_allreduce_kernel",        "proj_rowdot_kernel",
    "proj_colsum_kernel",       "proj_gemm_finish_kernel",      "complex_fwd_summary_kernel",
    "complex_carry_scan(fwd)",  "complex_fwd_replay_kernel",    "complex_bwd_summary_kernel",
    "complex_carry_scan(bwd)",  "complex_bwd_grad_kernel"};

cudaEvent_t take_event() {
  if (!g_pool.empty()) {
    cudaEvent_t e = g_pool.back();
    g_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return e;
}

}  // namespace

TimedLaunch::TimedLaunch(int id, cudaStream_t s) : id_(id), s_(s) {
  if (!g_on.load(std::memory_order_relaxed)) return;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  start_ = take_event();
  end_ = take_event();
  if (start_ == nullptr || end_ == nullptr || cudaEventRecord(start_, s) != cudaSuccess) {
    cudaGetLastError();
    if (start_) g_pool.push_back(start_);
    if (end_) g_pool.push_back(end_);
    start_ = end_ = nullptr;
  }
}

TimedLaunch::~TimedLaunch() {
  if (start_ == nullptr) return;
  std::lock_guard<std::mutex> lock(g_mu);
  if (cudaEventRecord(end_, s_) != cudaSuccess) {
    cudaGetLastError();
    g_pool.push_back(start_);
    g_pool.push_back(end_);
    return;
  }
  g_pending.push_back(Pending{id_, start_, end_});
}

}  // namespace sparc

using namespace sparc;

extern "C" {

int sparc_timing_enable(int on) { return g_on.exchange(on ? 1 : 0); }

const char* sparc_timing_kernel_name(int id) { return id >= 0 && id < kTimeKernels ? kNames[id] : ""; }

int sparc_timing_read(double* ms, long long* launches, int n) {
  std::lock_guard<std::mutex> lock(g_mu);
  for (const Pending& p : g_pending) {
    float t = 0.0f;
    if (cudaEventSynchronize(p.end) == cudaSuccess && cudaEventElapsedTime(&t, p.start, p.end) == cudaSuccess) {
      g_ms[p.id] += t;
      g_count[p.id] += 1;
    } else {
      cudaGetLastError();
    }
    g_pool.push_back(p.start);
    g_pool.push_back(p.end);
  }
  g_pending.clear();
  for (int i = 0; i < n && i < kTimeKernels; ++i) {
    if (ms) ms[i] = g_ms[i];
    if (launches) launches[i] = g_count[i];
  }
  for (int i = 0; i < kTimeKernels; ++i) {
    g_ms[i] = 0.0;
    g_count[i] = 0;
  }
  return kTimeKernels;
}

}  // extern "C"
