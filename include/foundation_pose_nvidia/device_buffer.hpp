// RAII device memory and streams (reference include/foundation_pose_nvidia/device_buffer.hpp:14-44).
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>

#include "foundation_pose_nvidia/exception.hpp"

#pragma GCC visibility push(default)
namespace foundation_pose_nvidia {

void checkCuda(cudaError_t status, const char* what);

class DeviceBuffer {
 public:
  DeviceBuffer() = default;
  explicit DeviceBuffer(std::size_t bytes) { allocate(bytes); }
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  DeviceBuffer(DeviceBuffer&& other) noexcept;
  DeviceBuffer& operator=(DeviceBuffer&& other) noexcept;
  ~DeviceBuffer();

  void allocate(std::size_t bytes);  // zero-filled
  void reset();
  void* data() { return ptr_; }
  const void* data() const { return ptr_; }
  std::size_t bytes() const { return bytes_; }
  template <class T>
  T* as() { return static_cast<T*>(ptr_); }
  template <class T>
  const T* as() const { return static_cast<const T*>(ptr_); }

 private:
  void* ptr_ = nullptr;
  std::size_t bytes_ = 0;
};

class CudaStream {
 public:
  explicit CudaStream(unsigned int flags = cudaStreamNonBlocking);
  CudaStream(const CudaStream&) = delete;
  CudaStream& operator=(const CudaStream&) = delete;
  CudaStream(CudaStream&& other) noexcept;
  CudaStream& operator=(CudaStream&& other) noexcept;
  ~CudaStream();
  cudaStream_t get() const { return stream_; }
  void synchronize() const;

 private:
  cudaStream_t stream_ = nullptr;
};

}  // namespace foundation_pose_nvidia
#pragma GCC visibility pop
