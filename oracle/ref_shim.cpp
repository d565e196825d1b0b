// ref_shim.cpp -- C entry points around the reference's own CPU scan.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's src/selective_scan.cpp, taken from where it lies in the
// reference checkout (never copied), into oracle/_ref/libref_scan.so.  The
// tests use it to pin the C restatement in oracle/scan_oracle.c, and bench.py
// uses it as the reference arm / CPU baseline ("kind": "reference").
//
// Wrapped interface: saccade::selective_scan_reference,
// include/saccade/selective_scan.hpp:38-39 (exceptions become return codes).
#include "saccade/selective_scan.hpp"

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <thread>
#include <vector>

namespace {
struct RefShape {
    std::uint64_t batch, length, channels, state, a_rows, c_width;
    std::int32_t has_d;
};

saccade::SelectiveScanShape to_shape(const RefShape& s) {
    saccade::SelectiveScanShape out;
    out.batch = s.batch;
    out.length = s.length;
    out.channels = s.channels;
    out.state = s.state;
    out.a_rows = s.a_rows;
    out.c_width = s.c_width;
    out.has_d = s.has_d != 0;
    return out;
}

void copy_message(char* msg, std::size_t cap, const char* text) {
    if (msg && cap) std::snprintf(msg, cap, "%s", text);
}
} // namespace

extern "C" {

// 0 = ok, 1 = std::invalid_argument, 2 = std::range_error, 3 = other exception.
int sacc_ref_selective_scan(const RefShape* s, const float* u, std::size_t n_u, const float* delta, std::size_t n_delta,
                            const float* a, std::size_t n_a, const float* b, std::size_t n_b, const float* c, std::size_t n_c,
                            const float* d, std::size_t n_d, double* y, char* msg, std::size_t cap) {
    try {
        const saccade::SelectiveScanInputs in{{u, n_u}, {delta, n_delta}, {a, n_a}, {b, n_b}, {c, n_c}, {d, n_d}};
        const auto out = saccade::selective_scan_reference(to_shape(*s), in);
        if (!out.empty()) std::memcpy(y, out.data(), out.size() * sizeof(double));
        return 0;
    } catch (const std::range_error& e) {
        copy_message(msg, cap, e.what());
        return 2;
    } catch (const std::invalid_argument& e) {
        copy_message(msg, cap, e.what());
        return 1;
    } catch (const std::exception& e) {
        copy_message(msg, cap, e.what());
        return 3;
    }
}

// The reference scan over a batch slice per host thread: batch rows are
// independent by contract (tests/selective_scan_tests.cpp:250-261), so each
// thread calls selective_scan_reference on a contiguous slice of rows.
// Returns the first non-zero status of any slice.
int sacc_ref_selective_scan_threads(const RefShape* s, const float* u, const float* delta, const float* a, const float* b,
                                    const float* c, const float* d, double* y, int threads) {
    const std::size_t B = s->batch, L = s->length, Dc = s->channels, N = s->state, cw = s->c_width;
    if (threads < 1) threads = 1;
    if (static_cast<std::size_t>(threads) > B) threads = static_cast<int>(B);
    std::vector<int> status(static_cast<std::size_t>(threads), 0);
    std::vector<std::thread> pool;
    for (int k = 0; k < threads; ++k) {
        const std::size_t b0 = B * k / threads, b1 = B * (k + 1) / threads;
        pool.emplace_back([=, &status] {
            RefShape part = *s;
            part.batch = b1 - b0;
            const std::size_t tok = b0 * L;
            status[static_cast<std::size_t>(k)] = sacc_ref_selective_scan(
                &part, u + tok * Dc, (b1 - b0) * L * Dc, delta + tok * Dc, (b1 - b0) * L * Dc, a, s->a_rows * N, b + tok * N,
                (b1 - b0) * L * N, c + tok * cw, (b1 - b0) * L * cw, d, s->has_d ? Dc : 0, y + tok * Dc, nullptr, 0);
        });
    }
    for (auto& t : pool) t.join();
    for (const int st : status)
        if (st) return st;
    return 0;
}

double sacc_ref_softplus(double x) { return saccade::selective_scan_softplus(x); }

} // extern "C"
