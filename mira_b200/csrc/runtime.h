// Host-side runtime shared by the entry points: per-device state (stream, SM count), the
// thread's last error message, argument checks and the kernel launch counter.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "../../include/mira_cuda.h"

namespace mira {

struct DeviceState {
  bool ready = false;
  int device = -1;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  cudaStream_t stream = nullptr;
  cudaStream_t copy_stream = nullptr;   // host<->device copies that overlap the kernels on `stream`
};

// State of the calling thread's current device (set up by mira_cuda_set_device; device 0 is
// selected on first use when the caller never chose one).
DeviceState* current_device();

int set_error(int code, const std::string& msg);
int cuda_error(cudaError_t e, const char* what);
void count_launch();

#define MIRA_CHECK_ARG(cond, msg) \
  do {                            \
    if (!(cond)) return ::mira::set_error(MIRA_CUDA_EINVAL, msg); \
  } while (0)

#define MIRA_CUDA_TRY(call, what)                    \
  do {                                               \
    cudaError_t e_ = (call);                         \
    if (e_ != cudaSuccess) return ::mira::cuda_error(e_, what); \
  } while (0)

// After a kernel launch: records a launch error, counts the launch.
int after_launch(const char* kernel);

// Fetches a device and fails if there is none.
#define MIRA_GET_DEVICE(dev)                                              \
  DeviceState* dev = ::mira::current_device();                            \
  if (dev == nullptr) return ::mira::set_error(MIRA_CUDA_ENODEV, "no usable CUDA device")

inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

}  // namespace mira
