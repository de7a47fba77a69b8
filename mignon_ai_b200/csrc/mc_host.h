// Host-side helpers of libmignoncuda: status/error reporting across the C-ABI and TMA tensor maps.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

namespace mc {

// Sets the thread-local message returned by mc_last_error() and returns status.
int set_error(int status, const std::string& msg);
void clear_error();

// Status codes of the C-ABI (mirrored in include/mignon_cuda.h).
enum Status : int {
  kOk = 0,
  kInvalidArgument = 1,
  kCudaError = 2,
  kBadModel = 3,
  kOutOfMemory = 4,
  kDeviceTimeout = 5,
  kUnsupported = 6,
};

// Checks a CUDA runtime call; on failure records the message and returns kCudaError.
#define MC_CUDA(call)                                                                         \
  do {                                                                                        \
    cudaError_t e_ = (call);                                                                  \
    if (e_ != cudaSuccess)                                                                    \
      return ::mc::set_error(::mc::kCudaError, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

// Encodes a 2-D tiled tensor map over a row-major int8 matrix [rows x cols] (cols contiguous,
// row pitch `pitch` bytes) with box {box_cols, box_rows} and the 128-byte swizzle. Returns false
// (with the error recorded) if the driver rejects it.
bool make_tmap_i8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch,
                  uint32_t box_cols, uint32_t box_rows);

// Reads and clears the device error word of the current device; non-zero codes become
// kDeviceTimeout with a message.
int check_device_error(cudaStream_t stream);

// Restores the calling thread's current CUDA device when the scope ends. Every entry point holds
// one: they switch to the devices of their shards, and the caller's own work afterwards (its
// kernels, or the _dev entry points on the default stream, which run on the current device) must
// still run on the device the caller chose.
struct DeviceRestore {
  int prev = -1;
  DeviceRestore() {
    if (cudaGetDevice(&prev) != cudaSuccess) {
      prev = -1;
      cudaGetLastError();
    }
  }
  ~DeviceRestore() {
    if (prev >= 0) cudaSetDevice(prev);
  }
  DeviceRestore(const DeviceRestore&) = delete;
  DeviceRestore& operator=(const DeviceRestore&) = delete;
};

}  // namespace mc
