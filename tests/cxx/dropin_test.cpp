// Compiled caller of the C++ drop-in (include/Kernels.hpp, include/Weight.hpp)
// that replays the reference engine's own GPU tests through this library:
//
//   src/tests/MatmulTests.cpp:12-82    three tensors, output overwritten on
//                                      reuse, two CudaStreams, zero input
//   src/tests/MatmulTests.cpp:84-132   dimension[1] narrowed to 19, rows
//                                      {1, 4, 5, 101}, 123.0f sentinels on
//                                      both sides of the product
//   src/tests/AttentionTests.cpp:9-74  the five causal GQA shapes, margin 3e-5
//
// plus the exception types of the reference API (std::invalid_argument for
// bad arguments: matmul.cu:132-136, rms_norm.cu:34-36, rope.cu:33-35,
// attention.cu:99-105, argmax.cu:72-74; std::runtime_error for CUDA
// failures: Kernels.hpp:14-33; std::logic_error for a moved-from
// CudaStream: CudaStream.cpp:33).
//
// The reference tests read a real GGUF model; here a stand-in model object
// serves seeded synthetic tensors of the same names and shapes (Qwen3-4B
// block 0: attn_q Q4_K 2560x4096, attn_v Q6_K 2560x1024, ffn_down Q6_K
// 9728x2560), through the get_tensor_info / read_tensor_data interface that
// Weight(model, name) uses. Expected products and attention outputs come
// from the CPU oracle (oracle/q4k_oracle.c: MatmulReference.hpp:42-64 and
// AttentionReference.hpp:13-88 restated). Test infrastructure only.
//
// Exit status 0 when every check passes; each failure is printed.
#include <array>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

#include "Kernels.hpp"
#include "q4k_oracle.h"

namespace {

int g_failures = 0;
int g_checks = 0;

void expect(bool ok, const std::string& what) {
    ++g_checks;
    if (!ok) {
        ++g_failures;
        std::printf("FAIL: %s\n", what.c_str());
    }
}

// Catch::Approx(expected).margin(m).epsilon(e) as the reference tests use it.
bool approx(double actual, double expected, double margin, double epsilon = 1e-4) {
    const double d = std::fabs(actual - expected);
    return d <= margin || d <= epsilon * std::fabs(expected);
}

// Stand-in for the reference's GGUF class: the two members Weight(model, name) calls.
class SyntheticModel {
public:
    struct TensorInfo {
        int type;
        std::array<int64_t, 4> dimensions;
    };

    void add(const std::string& name, int type, int64_t ne0, int64_t ne1) {
        const size_t block = type == ORC_Q4_K ? 144 : 210;
        std::vector<std::byte> bytes((size_t)ne1 * (size_t)(ne0 / 256) * block);
        if (orc_synth_tensor(0xD0C5ull, name.c_str(), type, ne0, ne1, bytes.data()) != 0)
            throw std::runtime_error("synthetic tensor " + name);
        info_[name] = TensorInfo{type, {ne0, ne1, 1, 1}};
        data_[name] = std::move(bytes);
    }
    const TensorInfo* get_tensor_info(const std::string& name) const { return &info_.at(name); }
    std::vector<std::byte> read_tensor_data(const std::string& name) const { return data_.at(name); }
    const std::byte* raw(const std::string& name) const { return data_.at(name).data(); }

private:
    std::map<std::string, TensorInfo> info_;
    std::map<std::string, std::vector<std::byte>> data_;
};

std::vector<float> make_input(size_t count) {  // MatmulReference.hpp:31-39
    std::vector<float> input(count);
    for (size_t i = 0; i < count; ++i) input[i] = std::sin(float(i) * 0.031f) * 0.1f;
    return input;
}

std::vector<double> expected_product(const SyntheticModel& model, const std::string& name, const Weight& weight,
                                     const std::vector<float>& input, size_t rows, size_t columns) {
    std::vector<double> y(rows * columns);
    const int rc = orc_matmul(input.data(), model.raw(name), weight.datatype, (size_t)weight.dimension[0], columns,
                              rows, y.data(), 0);
    if (rc != 0) throw std::runtime_error("oracle matmul " + name);
    return y;
}

void copy_to_host(const DeviceBuffer& source, std::vector<float>& destination) {
    expect(cudaMemcpy(destination.data(), source.data, destination.size() * sizeof(float), cudaMemcpyDeviceToHost) ==
               cudaSuccess,
           "device-to-host copy");
}

void require_product(const std::vector<float>& actual, const std::vector<double>& expected, size_t offset,
                     double margin, const std::string& what) {
    size_t bad = 0;
    double worst = 0.0;
    for (size_t i = 0; i < expected.size(); ++i) {
        if (!approx(actual[offset + i], expected[i], margin)) {
            ++bad;
            worst = std::fmax(worst, std::fabs(actual[offset + i] - expected[i]));
        }
    }
    expect(bad == 0, what + ": " + std::to_string(bad) + " of " + std::to_string(expected.size()) +
                         " outside the bar, worst |diff| " + std::to_string(worst));
}

template <class E, class F>
void expect_throw(F&& f, const std::string& what) {
    try {
        f();
        expect(false, what + ": no exception");
    } catch (const E&) {
        expect(true, what);
    } catch (const std::exception& e) {
        expect(false, what + ": wrong exception type (" + e.what() + ")");
    }
}

const char* const kNames[] = {"blk.0.attn_q.weight", "blk.0.attn_v.weight", "blk.0.ffn_down.weight"};

// MatmulTests.cpp:12-82
void matmul_overwrite_and_streams(const SyntheticModel& model) {
    for (const char* name : kNames) {
        const std::string tag = std::string("matmul/overwrite ") + name;
        Weight weight(model, name);
        expect(weight.datatype == (std::string(name) == "blk.0.attn_q.weight" ? GGML_TYPE_Q4_K : GGML_TYPE_Q6_K),
               tag + ": tensor type");
        const size_t width = weight.dimension[0];
        constexpr size_t columns = 5, rows = 3;
        weight.dimension[1] = columns;
        const auto input = make_input(rows * width);
        const auto expected = expected_product(model, name, weight, input, rows, columns);
        DeviceBuffer device_input(input.data(), input.size() * sizeof(float));
        std::vector<float> actual(rows * columns, 123.0f);
        DeviceBuffer device_output(actual.data(), actual.size() * sizeof(float));
        for (int repeat = 0; repeat < 2; ++repeat) {
            kernels::matmul(static_cast<const float*>(device_input.data), weight,
                            static_cast<float*>(device_output.data), rows);
            copy_to_host(device_output, actual);
            require_product(actual, expected, 0, 1e-5, tag + " repeat " + std::to_string(repeat));
        }
        DeviceBuffer other_output(actual.data(), actual.size() * sizeof(float));
        kernels::CudaStream first, second;
        kernels::matmul(static_cast<const float*>(device_input.data), weight, static_cast<float*>(device_output.data),
                        rows, first);
        kernels::matmul(static_cast<const float*>(device_input.data), weight, static_cast<float*>(other_output.data),
                        rows, second);
        first.synchronize();
        second.synchronize();
        for (const DeviceBuffer* buffer : {&device_output, &other_output}) {
            copy_to_host(*buffer, actual);
            require_product(actual, expected, 0, 1e-5, tag + " two streams");
        }
        expect(cudaMemset(device_input.data, 0, input.size() * sizeof(float)) == cudaSuccess, "memset");
        kernels::matmul(static_cast<const float*>(device_input.data), weight, static_cast<float*>(device_output.data),
                        1);
        expect(cudaMemcpy(actual.data(), device_output.data, columns * sizeof(float), cudaMemcpyDeviceToHost) ==
                   cudaSuccess,
               "copy");
        for (size_t i = 0; i < columns; ++i) expect(actual[i] == 0.0f, tag + ": zero input gives exact zeros");
    }
}

// MatmulTests.cpp:84-132
void matmul_row_counts(const SyntheticModel& model) {
    for (const char* name : kNames) {
        for (size_t rows : {size_t{1}, size_t{4}, size_t{5}, size_t{101}}) {
            const std::string tag = std::string("matmul/rows ") + name + " rows=" + std::to_string(rows);
            Weight weight(model, name);
            const size_t width = weight.dimension[0];
            constexpr size_t columns = 19;
            weight.dimension[1] = columns;
            const auto input = make_input(rows * width);
            const auto expected = expected_product(model, name, weight, input, rows, columns);
            DeviceBuffer device_input(input.data(), input.size() * sizeof(float));
            std::vector<float> actual(rows * columns + 2, 123.0f);
            DeviceBuffer output(actual.data(), actual.size() * sizeof(float));
            float* product = static_cast<float*>(output.data) + 1;
            kernels::CudaStream stream;
            for (int repeat = 0; repeat < 2; ++repeat) {
                kernels::matmul(static_cast<const float*>(device_input.data), weight, product, rows, stream);
                stream.synchronize();
                copy_to_host(output, actual);
                expect(actual.front() == 123.0f && actual.back() == 123.0f, tag + ": sentinels untouched");
                require_product(actual, expected, 1, 3e-5, tag);
            }
            expect(cudaMemset(device_input.data, 0, input.size() * sizeof(float)) == cudaSuccess, "memset");
            kernels::matmul(static_cast<const float*>(device_input.data), weight, product, rows);
            copy_to_host(output, actual);
            bool zeros = true;
            for (size_t i = 0; i < expected.size(); ++i) zeros = zeros && actual[i + 1] == 0.0f;
            expect(zeros, tag + ": zero input gives exact zeros");
        }
    }
}

// AttentionTests.cpp:9-74
void attention_shapes() {
    struct Shape {
        const char* name;
        size_t queries, prefix, heads, kv_heads, dim;
    };
    const Shape cases[] = {
        {"single value", 1, 0, 1, 1, 1},
        {"prefill with grouped query heads", 35, 0, 4, 2, 128},
        {"cached prefix with partial warp", 3, 31, 4, 1, 33},
        {"single token decode", 1, 64, 4, 2, 256},
        {"head dimension across tile boundary", 2, 32, 2, 2, 129},
    };
    for (const Shape& s : cases) {
        const size_t cached = s.prefix + s.queries;
        std::vector<float> q(s.queries * s.heads * s.dim), k(cached * s.kv_heads * s.dim), v(k.size());
        for (size_t i = 0; i < q.size(); ++i) q[i] = std::sin(float(i) * 0.13f) * 2.0f;
        for (size_t i = 0; i < k.size(); ++i) {
            k[i] = std::cos(float(i) * 0.07f) * 9.0f;
            v[i] = std::sin(float(i) * 0.11f);
        }
        std::vector<float> expected(q.size());
        expect(orc_attention(q.data(), k.data(), v.data(), expected.data(), s.queries, s.heads, s.kv_heads, s.dim,
                             s.prefix) == 0,
               "oracle attention");
        DeviceBuffer dq(q.data(), q.size() * sizeof(float));
        DeviceBuffer dk(k.data(), k.size() * sizeof(float));
        DeviceBuffer dv(v.data(), v.size() * sizeof(float));
        std::vector<float> actual(q.size() + 2, 123.0f);
        DeviceBuffer output(actual.data(), actual.size() * sizeof(float));
        for (int repeat = 0; repeat < 2; ++repeat) {
            kernels::attention(static_cast<const float*>(dq.data), static_cast<const float*>(dk.data),
                               static_cast<const float*>(dv.data), static_cast<float*>(output.data) + 1, s.queries,
                               s.heads, s.kv_heads, s.dim, s.prefix);
            copy_to_host(output, actual);
            expect(actual.front() == 123.0f && actual.back() == 123.0f, std::string("attention/") + s.name + ": sentinels");
            std::vector<double> want(expected.begin(), expected.end());
            require_product(actual, want, 1, 3e-5, std::string("attention/") + s.name);
        }
    }
}

// RMSNorm, RoPE, SiLU, residual add and argmax through the drop-in against
// the oracle, so that every kernels:: entry is called from C++.
void small_ops() {
    const size_t rows = 2, width = 2560;
    std::vector<float> x(rows * width), gamma(width), want(rows * width), got(rows * width);
    for (size_t i = 0; i < x.size(); ++i) x[i] = std::sin(float(i) * 0.017f) * 3.0f;
    for (size_t i = 0; i < width; ++i) gamma[i] = 1.0f + 0.01f * std::cos(float(i));
    Weight scale("output_norm.weight", GGML_TYPE_F32, {(int64_t)width}, gamma.data());
    DeviceBuffer dx(x.data(), x.size() * sizeof(float)), dy(x.size() * sizeof(float));
    kernels::rms_norm(static_cast<const float*>(dx.data), scale, static_cast<float*>(dy.data), rows, width, 1e-6f);
    copy_to_host(dy, got);
    orc_rms_norm(x.data(), gamma.data(), want.data(), rows, width, 1e-6f);
    std::vector<double> w(want.begin(), want.end());
    require_product(got, w, 0, 1e-6, "rms_norm");

    const size_t tokens = 3, heads = 4, dim = 128;
    std::vector<float> r(tokens * heads * dim), rw;
    for (size_t i = 0; i < r.size(); ++i) r[i] = std::cos(float(i) * 0.05f);
    rw = r;
    DeviceBuffer dr(r.data(), r.size() * sizeof(float));
    kernels::rope(static_cast<float*>(dr.data), tokens, heads, dim, 7, 1e6f);
    std::vector<float> rg(r.size());
    copy_to_host(dr, rg);
    orc_rope(rw.data(), tokens, heads, dim, 7, 1e6f);
    require_product(rg, std::vector<double>(rw.begin(), rw.end()), 0, 1e-4, "rope");

    std::vector<float> g(1000), u(1000), a(1000), b(1000);
    for (size_t i = 0; i < g.size(); ++i) {
        g[i] = std::sin(float(i) * 0.3f) * 4.0f;
        u[i] = std::cos(float(i) * 0.2f);
    }
    DeviceBuffer dg(g.data(), 4000), du(u.data(), 4000), da(4000);
    kernels::silu_multiply(static_cast<const float*>(dg.data), static_cast<const float*>(du.data),
                           static_cast<float*>(da.data), g.size());
    copy_to_host(da, a);
    orc_silu_multiply(g.data(), u.data(), b.data(), g.size());
    require_product(a, std::vector<double>(b.begin(), b.end()), 0, 1e-6, "silu_multiply");

    kernels::residual_add(static_cast<float*>(dg.data), static_cast<const float*>(du.data), g.size());
    copy_to_host(dg, a);
    orc_residual_add(g.data(), u.data(), g.size());
    bool same = true;
    for (size_t i = 0; i < g.size(); ++i) same = same && a[i] == g[i];
    expect(same, "residual_add bit-exact");

    std::vector<float> logits(151936);
    for (size_t i = 0; i < logits.size(); ++i) logits[i] = std::sin(float(i) * 0.001f);
    logits[123457] = 5.0f;
    logits[99] = 5.0f;  // tie: the lowest index wins (argmax.cu:25-61)
    DeviceBuffer dl(logits.data(), logits.size() * sizeof(float));
    expect(kernels::argmax(static_cast<const float*>(dl.data), logits.size()) == 99u, "argmax lowest index on ties");
}

void exceptions(const SyntheticModel& model) {
    std::vector<float> gamma(256, 1.0f);
    Weight f32("output_norm.weight", GGML_TYPE_F32, {256}, gamma.data());
    DeviceBuffer x(256 * sizeof(float)), y(4096 * sizeof(float));
    auto* xp = static_cast<const float*>(x.data);
    auto* yp = static_cast<float*>(y.data);
    expect_throw<std::invalid_argument>([&] { kernels::matmul(xp, f32, yp, 1); }, "matmul of an F32 weight");
    Weight q(model, "blk.0.attn_q.weight");
    q.dimension[0] = 100;
    expect_throw<std::invalid_argument>([&] { kernels::matmul(xp, q, yp, 1); }, "matmul with width % 256 != 0");
    q.dimension[0] = 2560;
    q.dimension[1] = 0;
    expect_throw<std::invalid_argument>([&] { kernels::matmul(xp, q, yp, 1); }, "matmul with no rows");
    expect_throw<std::invalid_argument>([&] { kernels::rms_norm(xp, f32, yp, 1, 128, 1e-6f); },
                                        "rms_norm with a scale of another width");
    expect_throw<std::invalid_argument>([&] { kernels::rms_norm(xp, f32, yp, 1, 256, 0.0f); },
                                        "rms_norm with epsilon 0");
    expect_throw<std::invalid_argument>([&] { kernels::rope(yp, 1, 1, 33, 0, 1e6f); }, "rope with an odd head_dim");
    expect_throw<std::invalid_argument>([&] { kernels::attention(xp, xp, xp, yp, 1, 3, 2, 16, 0); },
                                        "attention with heads not divisible by kv_heads");
    expect_throw<std::invalid_argument>([&] { kernels::attention(xp, xp, xp, yp, 1, 2, 2, 300, 0); },
                                        "attention with head_dim > 256");
    expect_throw<std::invalid_argument>([&] { kernels::argmax(xp, 0); }, "argmax of nothing");
    expect_throw<std::invalid_argument>([&] { DeviceBuffer b(nullptr, 16); }, "DeviceBuffer without host bytes");
    kernels::CudaStream s;
    kernels::CudaStream t(std::move(s));
    expect_throw<std::logic_error>([&] { (void)s.get(); }, "moved-from CudaStream");
    expect(t.ready(), "fresh stream is ready");
    // an allocation the device cannot satisfy: a CUDA error, reported as
    // std::runtime_error (no kernel runs)
    expect_throw<std::runtime_error>([&] { DeviceBuffer huge(size_t{1} << 52); }, "allocation beyond device memory");
    expect(kernels::detail::get_sm_count() > 0, "SM count");
}

}  // namespace

int main() {
    try {
        SyntheticModel model;
        model.add("blk.0.attn_q.weight", ORC_Q4_K, 2560, 4096);
        model.add("blk.0.attn_v.weight", ORC_Q6_K, 2560, 1024);
        model.add("blk.0.ffn_down.weight", ORC_Q6_K, 9728, 2560);
        matmul_overwrite_and_streams(model);
        matmul_row_counts(model);
        attention_shapes();
        small_ops();
        exceptions(model);
    } catch (const std::exception& e) {
        std::printf("FAIL: unexpected exception: %s\n", e.what());
        ++g_failures;
    }
    std::printf("%d checks, %d failures\n", g_checks, g_failures);
    return g_failures == 0 ? 0 : 1;
}
