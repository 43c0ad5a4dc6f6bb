// Calls the C++ boundary (include/axion_b200.hpp) the way the reference's
// runtime would, against the reference's own host path, in one process:
//   GGUFLoader::load_tensor + axion::linear_from_gguf   (the reference, CPU)
//   b200::load_tensor_raw + upload_q8_0 + b200::linear_from_gguf (device Q8_0)
// on the Q8_0 tensors of a GGUF file (argv[1]).  Test infrastructure: linked
// with the reference library built by oracle/Makefile.  Prints one line per
// check and "boundary ok" at the end; exit status 0 only if all checks pass.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "axion_b200.hpp"
#include "axq8.h"
#include "core/tensor_factory.hpp"
#include "gguf/gguf.hpp"
#include "runtime/linear.hpp"

using namespace axion;

static int failures = 0;

static void check(bool ok, const std::string& what) {
    std::printf("%s %s\n", ok ? "PASS" : "FAIL", what.c_str());
    if (!ok) failures++;
}

// max |y - ref| / (sum_k |x_k w_k|), the normalised error of the tests
static double rel_err(const float* y, const float* ref, const float* x, const float* w, int64_t M,
                      int64_t N, int64_t K) {
    double worst = 0.0;
    for (int64_t m = 0; m < M; m++)
        for (int64_t n = 0; n < N; n++) {
            double s = 0.0;
            for (int64_t k = 0; k < K; k++) s += std::fabs((double)x[m * K + k] * w[n * K + k]);
            const double e = std::fabs((double)y[m * N + n] - ref[m * N + n]) / (s + 1e-30);
            if (e > worst) worst = e;
        }
    return worst;
}

template <typename F>
static bool throws_with(F f, const char* text) {
    try {
        f();
    } catch (const std::runtime_error& e) {
        return std::strstr(e.what(), text) != nullptr;
    }
    return false;
}

int main(int argc, char** argv) {
    if (argc < 2) {
        std::fprintf(stderr, "usage: boundary_test model.gguf\n");
        return 2;
    }
    const std::string path = argv[1];
    GGUFLoader loader;
    loader.load_file(path);
    b200::DeviceAllocator& da = b200::DeviceAllocator::instance();
    const int64_t active0 = da.stats().active_allocations;
    uint32_t lcg = 12345u;
    auto rnd = [&] {
        lcg = lcg * 1664525u + 1013904223u;
        return ((float)(lcg >> 8) / 16777216.0f - 0.5f) * 4.0f;
    };
    for (const char* name : {"blk.0.ffn_up.weight", "blk.1.ffn_down.weight", "output.weight",
                             "blk.0.attn_k.weight"}) {
        Tensor wref = loader.load_tensor(name);               // reference dequant (fp32)
        b200::RawTensor raw = b200::load_tensor_raw(path, name);
        check(raw.shape == wref.shape && raw.type == 8, std::string(name) + ": raw shape/type");
        {
            Tensor wdev = b200::upload_q8_0(raw);
            check(b200::is_device_q8(wdev) && !b200::is_device_q8(wref),
                  std::string(name) + ": device Q8_0 recognised");
            const int64_t N = wdev.shape[0], K = wdev.shape[1];
            // device dequantization == GGUFLoader::load_tensor, bit for bit
            axq8_weight_t w{};
            axq8_weight_wrap(wdev.buffer->raw(), N, K, &w);
            AllocHandle dq = da.allocate(sizeof(float) * N * K, 256);
            std::vector<float> wd(N * K);
            axq8_dequantize(&w, static_cast<float*>(dq.ptr), nullptr);
            cudaMemcpy(wd.data(), dq.ptr, sizeof(float) * N * K, cudaMemcpyDeviceToHost);
            da.deallocate(dq);
            check(std::memcmp(wd.data(), wref.data(), sizeof(float) * N * K) == 0,
                  std::string(name) + ": device dequant == load_tensor");
            for (int64_t M : {1, 3, 16, 70}) {
                Tensor x = create_owned_tensor({M, K}, DType::FLOAT32);
                for (int64_t i = 0; i < M * K; i++) x.data()[i] = rnd();
                Tensor yref = axion::linear_from_gguf(x, wref);
                b200::set_activation_mode(AXQ8_ACT_F32);
                Tensor y32 = b200::linear_from_gguf(x, wdev);
                const double e32 = rel_err(y32.data(), yref.data(), x.data(), wref.data(), M, N, K);
                b200::set_activation_mode(AXQ8_ACT_Q8);
                Tensor y8 = b200::linear_from_gguf(x, wdev);
                const double e8 = rel_err(y8.data(), yref.data(), x.data(), wref.data(), M, N, K);
                char buf[160];
                std::snprintf(buf, sizeof buf, "%s M=%lld: A32 err %.2e, A8 err %.2e", name,
                              (long long)M, e32, e8);
                // A32 is the reference's arithmetic; A8 quantizes the input
                // (half a step, 1/254 of each 32-block's maximum, per element)
                check(e32 <= 1e-5 && e8 <= 5e-3 && y32.shape == yref.shape, buf);
                // device input -> device output from the same allocator
                Tensor xd = create_buffer_tensor({M, K}, DType::FLOAT32, &da);
                cudaMemcpy(xd.data(), x.data(), sizeof(float) * M * K, cudaMemcpyHostToDevice);
                Tensor yd = b200::linear_from_gguf(xd, wdev);
                std::vector<float> yh(M * N);
                cudaMemcpy(yh.data(), yd.data(), sizeof(float) * M * N, cudaMemcpyDeviceToHost);
                check(std::memcmp(yh.data(), y8.data(), sizeof(float) * M * N) == 0,
                      std::string(name) + ": device input == host input");
            }
            // the reference's errors, and a host weight refused
            Tensor bad = create_owned_tensor({2, K + 32}, DType::FLOAT32);
            check(throws_with([&] { b200::linear_from_gguf(bad, wdev); },
                              "linear_from_gguf dimension mismatch: input K != weight K"),
                  std::string(name) + ": K mismatch message");
            Tensor x1 = create_owned_tensor({1, K}, DType::FLOAT32);
            check(throws_with([&] { b200::linear_from_gguf(x1, wref); }, "not a device Q8_0"),
                  std::string(name) + ": host weight refused");
        }
    }
    check(throws_with([&] { b200::load_tensor_raw(path, "no.such.tensor"); }, "Tensor not found"),
          "missing tensor message");
    // every weight, input and output buffer went back to the allocator (the
    // per-thread staging of host inputs stays: two allocations)
    const int64_t active = da.stats().active_allocations - active0;
    check(active == 2, "device allocations released (staging only): " + std::to_string(active));
    int status = 0;
    axq8_status_read(&status);
    check(status == 0, "device status word");
    std::printf(failures ? "boundary FAILED (%d)\n" : "boundary ok\n", failures);
    return failures ? 1 : 0;
}
