// C++ face of the B200 Q8_0 linear path for the reference's runtime
// (include/axion_b200.hpp): a device IAllocator, raw GGUF tensor reads, the
// one-time Q8_0 upload into a runtime Tensor, and linear_from_gguf on a device
// Q8_0 weight.  Host code only; the device work goes through the C ABI of
// libaxq8.so (include/axq8.h).  Compiled against the reference's headers.
#include "axion_b200.hpp"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <fstream>
#include <stdexcept>

#include "axq8.h"
#include "core/tensor_factory.hpp"

namespace axion {
namespace b200 {

namespace {

[[noreturn]] void throw_cuda(cudaError_t e, const char* what) {
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

[[noreturn]] void throw_axq8(int rc, const char* what) {
    throw std::runtime_error(std::string(what) + ": " + axq8_last_error() + " (status " +
                             std::to_string(rc) + ")");
}

// Device Q8_0 weights made by upload_q8_0: device address -> [N, K].
struct Q8Entry {
    int64_t N, K;
};
std::mutex g_q8_mu;
std::unordered_map<const void*, Q8Entry> g_q8;

int g_act_mode = AXQ8_ACT_Q8;

bool on_device(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        (void)cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice;
}

// Per-thread staging of host inputs and outputs (grow-only, device memory).
struct Staging {
    AllocHandle x, y;
    ~Staging() {
        DeviceAllocator::instance().deallocate(x);
        DeviceAllocator::instance().deallocate(y);
    }
    void* get(AllocHandle& h, size_t bytes) {
        if (h.bytes < bytes) {
            DeviceAllocator::instance().deallocate(h);
            h = DeviceAllocator::instance().allocate(bytes, 256);
        }
        return h.ptr;
    }
};

// ---- GGUF v3 directory -------------------------------------------------------
// Reads the header, skips the key/value section (keeping general.alignment),
// then walks the tensor infos; every integer is little-endian.
class Reader {
public:
    explicit Reader(const std::string& path) : f_(path, std::ios::binary) {
        if (!f_) throw std::runtime_error("Failed to open GGUF file: " + path);
    }
    template <typename T>
    T get() {
        T v;
        f_.read(reinterpret_cast<char*>(&v), sizeof(T));
        if (!f_) throw std::runtime_error("GGUF: unexpected end of file");
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (n > (1ull << 30)) throw std::runtime_error("GGUF: string too long");
        std::string s(n, '\0');
        f_.read(&s[0], (std::streamsize)n);
        if (!f_) throw std::runtime_error("GGUF: unexpected end of file");
        return s;
    }
    void skip(uint64_t n) { f_.seekg((std::streamoff)n, std::ios::cur); }
    uint64_t tell() { return (uint64_t)f_.tellg(); }
    void seek(uint64_t off) { f_.seekg((std::streamoff)off, std::ios::beg); }
    void read(void* dst, size_t n) {
        f_.read(static_cast<char*>(dst), (std::streamsize)n);
        if (!f_) throw std::runtime_error("GGUF: unexpected end of file");
    }

private:
    std::ifstream f_;
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case 0: case 1: case 7: return 1;             // u8, i8, bool
        case 2: case 3: return 2;                     // u16, i16
        case 4: case 5: case 6: return 4;             // u32, i32, f32
        case 10: case 11: case 12: return 8;          // u64, i64, f64
        default: return 0;                            // string (8), array (9)
    }
}

// Skip one value of type t; returns it when it is an unsigned 32-bit integer.
uint64_t skip_value(Reader& r, uint32_t t) {
    if (t == 8) {
        r.str();
        return 0;
    }
    if (t == 9) {
        const uint32_t et = r.get<uint32_t>();
        const uint64_t n = r.get<uint64_t>();
        for (uint64_t i = 0; i < n; i++) {
            if (scalar_size(et)) r.skip(scalar_size(et));
            else skip_value(r, et);
        }
        return 0;
    }
    if (t == 4) return r.get<uint32_t>();
    const size_t sz = scalar_size(t);
    if (!sz) throw std::runtime_error("GGUF: unknown metadata type " + std::to_string(t));
    r.skip(sz);
    return 0;
}

uint64_t type_bytes(uint32_t type, uint64_t n) {
    switch (type) {
        case 0: return n * 4;                          // F32
        case 1: return n * 2;                          // F16
        case 8: return axq8_q8_0_byte_size(n);         // Q8_0: (n / 32) * 34
        default:
            throw std::runtime_error("GGUF: tensor type " + std::to_string(type) +
                                     " not supported by load_tensor_raw (F32, F16, Q8_0)");
    }
}

}  // namespace

// ---- DeviceAllocator -----------------------------------------------------------

AllocHandle DeviceAllocator::allocate(size_t bytes, size_t alignment) {
    AllocHandle h;
    if (alignment > 256 || (alignment & (alignment - 1)))
        throw std::runtime_error("b200-device allocator: alignment must be a power of two <= 256");
    void* p = nullptr;
    const cudaError_t e = cudaMalloc(&p, bytes ? bytes : 1);   // 256-byte aligned
    if (e != cudaSuccess) throw_cuda(e, "b200-device allocator: cudaMalloc");
    std::lock_guard<std::mutex> lk(mu_);
    h.ptr = p;
    h.bytes = bytes;
    h.alignment = alignment ? alignment : kDefaultAlignment;
    h.id = next_id_++;
    stats_.allocated_bytes += (int64_t)bytes;
    stats_.peak_bytes = std::max(stats_.peak_bytes, stats_.allocated_bytes);
    stats_.allocation_count++;
    stats_.active_allocations++;
    return h;
}

void DeviceAllocator::deallocate(AllocHandle& h) {
    if (!h.valid()) return;
    {
        std::lock_guard<std::mutex> lk(g_q8_mu);
        g_q8.erase(h.ptr);
    }
    cudaFree(h.ptr);
    std::lock_guard<std::mutex> lk(mu_);
    stats_.allocated_bytes -= (int64_t)h.bytes;
    stats_.active_allocations--;
    h = AllocHandle{};
}

AllocatorStats DeviceAllocator::stats() const {
    std::lock_guard<std::mutex> lk(mu_);
    return stats_;
}

const char* DeviceAllocator::name() const { return "b200-device"; }

DeviceAllocator& DeviceAllocator::instance() {
    static DeviceAllocator* a = new DeviceAllocator();   // outlives static Tensors
    return *a;
}

// ---- raw tensors and upload ------------------------------------------------------

RawTensor load_tensor_raw(const std::string& path, const std::string& name) {
    Reader r(path);
    if (r.get<uint32_t>() != 0x46554747u) throw std::runtime_error("Invalid GGUF magic");
    const uint32_t version = r.get<uint32_t>();
    if (version < 2) throw std::runtime_error("GGUF: version " + std::to_string(version));
    const uint64_t n_tensors = r.get<uint64_t>();
    const uint64_t n_kv = r.get<uint64_t>();
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv; i++) {
        const std::string key = r.str();
        const uint32_t t = r.get<uint32_t>();
        const uint64_t v = skip_value(r, t);
        if (key == "general.alignment" && t == 4 && v) alignment = v;
    }
    RawTensor out;
    uint64_t offset = 0, count = 0;
    bool found = false;
    for (uint64_t i = 0; i < n_tensors; i++) {
        const std::string tn = r.str();
        const uint32_t nd = r.get<uint32_t>();
        std::vector<int64_t> dims(nd);
        for (uint32_t d = 0; d < nd; d++) dims[d] = (int64_t)r.get<uint64_t>();
        const uint32_t type = r.get<uint32_t>();
        const uint64_t off = r.get<uint64_t>();
        if (tn == name) {
            found = true;
            out.name = tn;
            out.type = type;
            out.shape.assign(dims.rbegin(), dims.rend());   // GGML order is inner first
            count = 1;
            for (int64_t d : dims) count *= (uint64_t)d;
            offset = off;
        }
    }
    if (!found) throw std::runtime_error("Tensor not found");
    const uint64_t data0 = (r.tell() + alignment - 1) / alignment * alignment;
    out.bytes.resize(type_bytes(out.type, count));
    r.seek(data0 + offset);
    r.read(out.bytes.data(), out.bytes.size());
    return out;
}

Tensor upload_q8_0(const RawTensor& raw) {
    if (raw.type != 8 || raw.shape.size() != 2)
        throw std::runtime_error("upload_q8_0: '" + raw.name + "' is not a 2-D Q8_0 tensor");
    const int64_t N = raw.shape[0], K = raw.shape[1];
    if (K % 32 || (uint64_t)raw.bytes.size() != axq8_q8_0_byte_size((uint64_t)(N * K)))
        throw std::runtime_error("upload_q8_0: '" + raw.name + "' has an inconsistent size");
    DeviceAllocator& da = DeviceAllocator::instance();
    Tensor t;
    t.name = raw.name;
    t.dtype = DType::UNKNOWN;
    t.shape = {N, K};
    t.storage = TensorStorage::BUFFER;
    t.buffer = TensorBuffer::create(da, (size_t)N * axq8_row_stride(K), 256);
    t.data_ptr = t.buffer->data();
    AllocHandle staging = da.allocate(raw.bytes.size(), 256);
    cudaError_t e = cudaMemcpy(staging.ptr, raw.bytes.data(), raw.bytes.size(), cudaMemcpyHostToDevice);
    int rc = e == cudaSuccess ? axq8_weight_repack(staging.ptr, N, K, t.buffer->raw(), nullptr) : AXQ8_OK;
    if (e == cudaSuccess && rc == AXQ8_OK) e = cudaDeviceSynchronize();
    da.deallocate(staging);
    if (e != cudaSuccess) throw_cuda(e, "upload_q8_0");
    if (rc != AXQ8_OK) throw_axq8(rc, "upload_q8_0");
    std::lock_guard<std::mutex> lk(g_q8_mu);
    g_q8[t.buffer->raw()] = Q8Entry{N, K};
    return t;
}

bool is_device_q8(const Tensor& t) {
    if (t.storage != TensorStorage::BUFFER || !t.buffer || t.shape.size() != 2) return false;
    std::lock_guard<std::mutex> lk(g_q8_mu);
    auto it = g_q8.find(t.buffer->raw());
    return it != g_q8.end() && it->second.N == t.shape[0] && it->second.K == t.shape[1];
}

void set_activation_mode(int act_mode) {
    if (act_mode != AXQ8_ACT_Q8 && act_mode != AXQ8_ACT_F32)
        throw std::runtime_error("set_activation_mode: AXQ8_ACT_Q8 or AXQ8_ACT_F32");
    g_act_mode = act_mode;
}

int activation_mode() { return g_act_mode; }

// ---- linear_from_gguf on a device Q8_0 weight --------------------------------------

Tensor linear_from_gguf(const Tensor& input, const Tensor& weight) {
    // the reference's argument checks and messages (linear.cpp:31-44)
    if (input.shape.size() != 2 || weight.shape.size() != 2)
        throw std::runtime_error("linear_from_gguf expects 2D input [M,K] and weight [N,K]");
    const int64_t M = input.shape[0], K = input.shape[1], N = weight.shape[0];
    if (K != weight.shape[1])
        throw std::runtime_error("linear_from_gguf dimension mismatch: input K != weight K");
    if (!is_device_q8(weight))
        throw std::runtime_error("linear_from_gguf: weight '" + weight.name +
                                 "' is not a device Q8_0 tensor (make it with upload_q8_0)");
    if (input.dtype != DType::FLOAT32)
        throw std::runtime_error("linear_from_gguf: input must be FLOAT32");
    axq8_weight_t w{};
    int rc = axq8_weight_wrap(const_cast<Tensor&>(weight).buffer->raw(), N, K, &w);
    if (rc) throw_axq8(rc, "linear_from_gguf");
    const float* x = input.data();
    if (M == 0) return on_device(x) ? create_buffer_tensor({0, N}, DType::FLOAT32, &DeviceAllocator::instance())
                                    : create_owned_tensor({0, N}, DType::FLOAT32);
    if (on_device(x)) {
        Tensor out = create_buffer_tensor({M, N}, DType::FLOAT32, &DeviceAllocator::instance());
        out.name = "linear_from_gguf_output";
        if ((rc = axq8_linear(&w, x, M, out.data(), g_act_mode, nullptr))) throw_axq8(rc, "linear_from_gguf");
        const cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) throw_cuda(e, "linear_from_gguf");
        return out;
    }
    thread_local Staging st;
    float* xd = static_cast<float*>(st.get(st.x, sizeof(float) * (size_t)(M * K)));
    float* yd = static_cast<float*>(st.get(st.y, sizeof(float) * (size_t)(M * N)));
    Tensor out = create_owned_tensor({M, N}, DType::FLOAT32);
    out.name = "linear_from_gguf_output";
    cudaError_t e = cudaMemcpy(xd, x, sizeof(float) * (size_t)(M * K), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) throw_cuda(e, "linear_from_gguf: input copy");
    if ((rc = axq8_linear(&w, xd, M, yd, g_act_mode, nullptr))) throw_axq8(rc, "linear_from_gguf");
    e = cudaMemcpy(out.data(), yd, sizeof(float) * (size_t)(M * N), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) throw_cuda(e, "linear_from_gguf: output copy");
    return out;
}

}  // namespace b200
}  // namespace axion
