// ref_head_shim.cpp -- C entry points around the reference's own binary64
// Mamba head (src/head_reference.cpp).
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's src/head_reference.cpp, src/head_weights.cpp,
// src/torch_checkpoint.cpp, src/sha256.cpp and src/file_io.cpp, taken from
// where they lie in the reference checkout (never copied), into
// oracle/_ref/libref_head.so.  The CPU tests use it to pin the block oracle
// (oracle/mamba_oracle.py) to the reference's arithmetic; the golden
// generator (tests/golden/make_head_golden.py) records its outputs.
//
// Wrapped interfaces (include/saccade/head_reference.hpp):
//   head_reference (:89-91) with keep_intermediates: the complete head on
//     synthetic_head_weights(seed) (:127) and head_test_features (:123-124),
//     every intermediate of a level kept ("p3.tokens", "p3.residual", ...);
//   head_ref::linear (:103), causal_conv1d (:105), silu (:106), multiply
//     (:107), add (:108), selective_scan (:119-120) on caller data: FP32
//     inputs widened exactly, or binary64 inputs (value only; bound and scale 0).
// Every function returns 0, or -1 with the exception's text in msg.
#include "saccade/head_reference.hpp"

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <exception>
#include <map>
#include <mutex>
#include <span>
#include <string>
#include <vector>

namespace {
using saccade::HeadReferenceResult;
using saccade::HeadTensor;
using saccade::HeadTensorRef;

void copy_message(char* msg, std::size_t cap, const char* text) {
    if (msg && cap) std::snprintf(msg, cap, "%s", text);
}

template <typename F>
int guarded(char* msg, std::size_t cap, F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        copy_message(msg, cap, e.what());
    } catch (...) {
        copy_message(msg, cap, "unknown exception");
    }
    return -1;
}

std::size_t count(const std::vector<std::int64_t>& shape) {
    std::size_t n = 1;
    for (const auto d : shape) n *= static_cast<std::size_t>(d);
    return n;
}

// A binary64 input with zero bound and scale (head_ref::from_float for FP32 data).
HeadTensorRef ref_of(const double* values, std::vector<std::int64_t> shape) {
    const auto n = count(shape);
    HeadTensorRef t{std::move(shape), std::vector<double>(values, values + n), std::vector<double>(n, 0.0),
                    std::vector<double>(n, 0.0)};
    return t;
}

HeadTensor weight_of(const float* values, std::vector<std::int64_t> shape) {
    const auto n = count(shape);
    return HeadTensor{std::move(shape), std::vector<float>(values, values + n)};
}

void put(const HeadTensorRef& t, double* value, double* sigma) {
    std::copy(t.value.begin(), t.value.end(), value);
    if (sigma) std::copy(t.sigma.begin(), t.sigma.end(), sigma);
}

// The last complete-head run, kept for the tensor queries below.
std::mutex g_mu;
HeadReferenceResult g_result;
saccade::HeadWeights g_weights;
} // namespace

extern "C" {

// Runs the reference's complete head (all three levels) on
// synthetic_head_weights(weight_seed) and head_test_features(kind,
// feature_seed, profile) (profile 0: T01 640x640, 1: HR 1280x768), keeping the
// intermediates for sacc_ref_head_tensor.
int sacc_ref_head_run(std::uint64_t weight_seed, const char* kind, std::uint64_t feature_seed, int profile, char* msg,
                      std::size_t cap) {
    return guarded(msg, cap, [&] {
        const auto prof = profile == 1 ? saccade::ModelProfile::Hr1280x768 : saccade::ModelProfile::T01_640x640;
        auto weights = saccade::synthetic_head_weights(weight_seed);
        const auto features = saccade::head_test_features(kind, feature_seed, prof);
        const std::array<std::span<const float>, 3> spans{std::span<const float>(features[0]), std::span<const float>(features[1]),
                                                          std::span<const float>(features[2])};
        auto result = saccade::head_reference(weights, spans, {}, true, prof);
        std::lock_guard lock(g_mu);
        g_result = std::move(result);
        g_weights = std::move(weights);
    });
}

// Shape (rank, up to 4 dims) and, when value is non-null, the values and
// scales of intermediate `name` of the last run ("p5.tokens", ...).
int sacc_ref_head_tensor(const char* name, std::int64_t* shape, int* rank, double* value, double* sigma, char* msg,
                         std::size_t cap) {
    return guarded(msg, cap, [&] {
        std::lock_guard lock(g_mu);
        for (const auto& [key, t] : g_result.intermediates) {
            if (key != name) continue;
            *rank = static_cast<int>(t.shape.size());
            for (std::size_t i = 0; i < t.shape.size() && i < 4; ++i) shape[i] = t.shape[i];
            if (value) put(t, value, sigma);
            return;
        }
        throw std::invalid_argument(std::string("no intermediate named ") + name);
    });
}

// Shape and FP32 values of parameter `name` of the last run's weights
// ("p5.mamba.in_proj.weight", ...).
int sacc_ref_head_weight(const char* name, std::int64_t* shape, int* rank, float* values, char* msg, std::size_t cap) {
    return guarded(msg, cap, [&] {
        std::lock_guard lock(g_mu);
        const auto& t = g_weights.at(name);
        *rank = static_cast<int>(t.shape.size());
        for (std::size_t i = 0; i < t.shape.size() && i < 4; ++i) shape[i] = t.shape[i];
        if (values) std::copy(t.values.begin(), t.values.end(), values);
    });
}

// head_ref::linear: x (rows, in) binary64, w (out, in) FP32, optional bias (out).
int sacc_ref_head_linear(const double* x, std::int64_t rows, std::int64_t in, const float* w, std::int64_t out,
                         const float* bias, double* y, double* sigma, char* msg, std::size_t cap) {
    return guarded(msg, cap, [&] {
        const auto wt = weight_of(w, {out, in});
        const HeadTensor bt = bias ? weight_of(bias, {out}) : HeadTensor{};
        put(saccade::head_ref::linear(ref_of(x, {rows, in}), wt, bias ? &bt : nullptr), y, sigma);
    });
}

// head_ref::causal_conv1d: x (B, L, C) binary64, w (C, 1, K), bias (C) FP32.
int sacc_ref_head_causal_conv1d(const double* x, std::int64_t batch, std::int64_t length, std::int64_t channels,
                                const float* w, std::int64_t k, const float* bias, double* y, char* msg, std::size_t cap) {
    return guarded(msg, cap, [&] {
        put(saccade::head_ref::causal_conv1d(ref_of(x, {batch, length, channels}), weight_of(w, {channels, 1, k}),
                                             weight_of(bias, {channels})),
            y, nullptr);
    });
}

int sacc_ref_head_silu(const double* x, std::int64_t n, double* y, char* msg, std::size_t cap) {
    return guarded(msg, cap, [&] { put(saccade::head_ref::silu(ref_of(x, {n})), y, nullptr); });
}

int sacc_ref_head_multiply(const double* a, const double* b, std::int64_t n, double* y, char* msg, std::size_t cap) {
    return guarded(msg, cap, [&] { put(saccade::head_ref::multiply(ref_of(a, {n}), ref_of(b, {n})), y, nullptr); });
}

int sacc_ref_head_add(const double* a, const double* b, std::int64_t n, double* y, char* msg, std::size_t cap) {
    return guarded(msg, cap, [&] { put(saccade::head_ref::add(ref_of(a, {n}), ref_of(b, {n})), y, nullptr); });
}

// head_ref::selective_scan: u, delta (B, L, Dc), A (1, N), B (B, L, N), C
// (B, L, 1) binary64; D (Dc) FP32 or null.  y (B, L, Dc) and its scale.
int sacc_ref_head_selective_scan(const double* u, const double* delta, const double* a, const double* b, const double* c,
                                 const float* d, std::int64_t batch, std::int64_t length, std::int64_t channels,
                                 std::int64_t state, double* y, double* sigma, char* msg, std::size_t cap) {
    return guarded(msg, cap, [&] {
        const HeadTensor dt = d ? weight_of(d, {channels}) : HeadTensor{};
        put(saccade::head_ref::selective_scan(ref_of(u, {batch, length, channels}), ref_of(delta, {batch, length, channels}),
                                              ref_of(a, {1, state}), ref_of(b, {batch, length, state}),
                                              ref_of(c, {batch, length, 1}), d ? &dt : nullptr),
            y, sigma);
    });
}

double sacc_ref_head_softplus(double x) { return saccade::head_ref::softplus(x); }

} // extern "C"
