// axion_b200.hpp — C++ face of the B200 Q8_0 linear path for the reference's
// runtime (namespace axion), built on the C ABI of axq8.h.
//
// This header is compiled INSIDE the reference's source tree: it includes the
// reference's own core/tensor.hpp, core/allocator.hpp and core/tensor_buffer.hpp
// (add inference/cpp to the include path), and the objects it declares are
// that runtime's Tensor and IAllocator, so the loader, the executor and the
// bindings can hand them to the device path unchanged.
//
// Reference interfaces it extends (paths inside the reference project):
//   IAllocator (byte allocator boundary)     inference/cpp/core/allocator.hpp:41-62
//   TensorBuffer / create_buffer_tensor      inference/cpp/core/tensor_buffer.hpp,
//                                            core/tensor_factory.hpp
//   GGUFLoader::load_tensor (Q8_0 branch)    inference/cpp/gguf/gguf.hpp:92-94,
//                                            gguf.cpp:784-882
//   linear_from_gguf                         inference/cpp/runtime/linear.hpp:22-25
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "core/allocator.hpp"
#include "core/tensor.hpp"
#include "core/tensor_buffer.hpp"

namespace axion {
namespace b200 {

// IAllocator over device memory of the current CUDA device (cudaMalloc,
// alignment up to 256 bytes).  Tensors made with create_buffer_tensor(shape,
// dtype, &DeviceAllocator::instance()) live in HBM: their data() pointer is a
// device address, which the host must not dereference.  Thread-safe.
class DeviceAllocator : public IAllocator {
public:
    AllocHandle allocate(size_t bytes, size_t alignment = kDefaultAlignment) override;
    void deallocate(AllocHandle& handle) override;
    AllocatorStats stats() const override;
    const char* name() const override;   // "b200-device"
    static DeviceAllocator& instance();

private:
    mutable std::mutex mu_;
    AllocatorStats stats_;
    uint64_t next_id_ = 1;
};

// One GGUF tensor's bytes as stored in the file, without dequantization:
// type is the GGUF/ggml type id (8 = Q8_0, 0 = F32), shape row-major
// [outer, ..., inner] as GGUFLoader reports it.
struct RawTensor {
    std::string name;
    uint32_t type = 0;
    std::vector<int64_t> shape;
    std::vector<uint8_t> bytes;
};

// GGUFLoader::load_tensor without the Q8_0 -> fp32 dequantization: the raw
// blocks of `name` from the GGUF v3 file at `path` (same directory rules: GGML
// dims reversed, data section aligned to general.alignment, default 32).
// Throws std::runtime_error("Tensor not found") like the loader.
RawTensor load_tensor_raw(const std::string& path, const std::string& name);

// Upload a Q8_0 tensor ([N, K], K % 32 == 0) once into device memory, in the
// repacked row layout of axq8.h, as a Tensor the runtime can hold: shape
// {N, K}, dtype UNKNOWN (the runtime has no Q8_0 dtype), storage BUFFER with a
// TensorBuffer from DeviceAllocator (freed with the last Tensor copy).
Tensor upload_q8_0(const RawTensor& raw);

// Whether t is a device Q8_0 weight made by upload_q8_0.
bool is_device_q8(const Tensor& t);

// Activation handling of linear_from_gguf (process-wide, default A8):
// AXQ8_ACT_Q8 quantizes each 32-block of the input (the decode default),
// AXQ8_ACT_F32 keeps fp32 activations (the reference's arithmetic).
void set_activation_mode(int act_mode);
int activation_mode();

// linear_from_gguf(input [M, K] fp32, weight [N, K] device Q8_0) -> [M, N]:
// the reference's operator with the weight resident in HBM.  A host input
// (owned or buffer-backed fp32) gives a new owned host output (copies in and
// out on the calling thread's stream, synchronized before return); a device
// input (created with DeviceAllocator) gives a device output from the same
// allocator.  Same argument checks and messages as the reference; throws
// std::runtime_error on any failure (the C ABI's message appended).
Tensor linear_from_gguf(const Tensor& input, const Tensor& weight);

}  // namespace b200
}  // namespace axion
