/*
 * scan_oracle.c -- CPU restatement (binary64) of the reference selective scan.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker, never the product:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm may load it.  The CUDA library under saccade_v1_b200/ never links it and
 * never falls back to it.
 *
 * Every function cites the reference file:line (paths relative to the
 * saccade_v1 project root) whose behaviour it restates.  Parity of this
 * restatement is pinned in tests/test_oracle.py against
 *   - the bc-derived closed forms of fixtures/selective-scan/expected.tsv
 *     (copied as tests/golden/scan_expected.json by tests/golden/make_golden.py),
 *   - outputs of the reference's own selective_scan_reference built from its
 *     sources into oracle/_ref/ (see oracle/Makefile), on seeded random cases.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, so that every binary64
 * product and sum rounds exactly where the reference's does).
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#define ORACLE_OK 0
#define ORACLE_INVALID 1
#define ORACLE_RANGE 2

/* src/selective_scan.cpp:15 -- the deployed kernel indexes with int32. */
static const size_t kMaxElements = 2147483647u;
/* src/selective_scan.cpp:16 */
static const double kFp32Max = 3.4028234663852886e38;

typedef struct {
    uint64_t batch, length, channels, state, a_rows, c_width;
    int32_t has_d;
} OracleShape;

static int fail(char* msg, size_t cap, int code, const char* text) {
    if (msg && cap) snprintf(msg, cap, "%s", text);
    return code;
}

/* src/selective_scan.cpp:59 -- threshold 20, log1p(exp(x)) below it. */
double sacc_oracle_softplus(double x) { return x > 20.0 ? x : log1p(exp(x)); }

/* src/selective_scan.cpp:20-28: product of dims with an int32 capacity check. */
static int elements(const uint64_t* dims, int n, size_t* out) {
    size_t product = 1;
    for (int i = 0; i < n; ++i) {
        if (dims[i] != 0 && product > kMaxElements / dims[i]) return 0;
        product *= dims[i];
    }
    *out = product;
    return 1;
}

static int is_finite_f(float v) { return isfinite(v); }

/* src/selective_scan.cpp:35-38 */
static int expect_finite(const float* v, size_t n, const char* name, char* msg, size_t cap) {
    for (size_t i = 0; i < n; ++i)
        if (!is_finite_f(v[i])) {
            if (msg && cap) snprintf(msg, cap, "selective_scan: %s[%zu] is not finite", name, i);
            return 0;
        }
    return 1;
}

/* src/selective_scan.cpp:40-45 */
static int in_range(double value, const char* quantity, size_t b, size_t t, size_t d, char* msg, size_t cap) {
    if (!(fabs(value) <= kFp32Max)) {
        if (msg && cap)
            snprintf(msg, cap, "selective_scan: %s leaves FP32 range at batch %zu, token %zu, channel %zu", quantity, b, t, d);
        return 0;
    }
    return 1;
}

/*
 * src/selective_scan.cpp:61-109 (selective_scan_reference).
 * Tensors are dense row-major FP32 with the reference ABI layouts:
 *   u, delta, y: (batch, length, channels); a: (a_rows, state);
 *   b: (batch, length, state); c: (batch, length, c_width); d: (channels).
 * The n_* arguments are the caller's element counts (the reference's spans).
 * Returns ORACLE_OK, ORACLE_INVALID (std::invalid_argument) or ORACLE_RANGE
 * (std::range_error) with the reference's diagnostic text in msg.
 */
int sacc_oracle_scan_ref(const OracleShape* s, const float* u, size_t n_u, const float* delta, size_t n_delta,
                         const float* a, size_t n_a, const float* b, size_t n_b, const float* c, size_t n_c,
                         const float* d, size_t n_d, double* y, char* msg, size_t cap) {
    char text[256];
    if (s->batch == 0 || s->channels == 0) return fail(msg, cap, ORACLE_INVALID, "selective_scan: batch and channels must be positive");
    if (s->state == 0 || s->state > 32 || (s->state & (s->state - 1)) != 0) {
        snprintf(text, sizeof text, "selective_scan: state %llu must be a power of two in [1, 32]", (unsigned long long)s->state);
        return fail(msg, cap, ORACLE_INVALID, text);
    }
    if (s->a_rows != 1 && s->a_rows != s->channels) return fail(msg, cap, ORACLE_INVALID, "selective_scan: A rows must be 1 or channels");
    if (s->c_width != 1 && s->c_width != s->state) return fail(msg, cap, ORACLE_INVALID, "selective_scan: C width must be 1 or state");
    size_t ud, bn, cn, an;
    const uint64_t d_ud[3] = {s->batch, s->length, s->channels}, d_bn[3] = {s->batch, s->length, s->state},
                   d_cn[3] = {s->batch, s->length, s->c_width}, d_an[2] = {s->a_rows, s->state};
    if (!elements(d_ud, 3, &ud)) return fail(msg, cap, ORACLE_INVALID, "selective_scan: u/delta/y element count exceeds int32 capacity");
    if (!elements(d_bn, 3, &bn)) return fail(msg, cap, ORACLE_INVALID, "selective_scan: B element count exceeds int32 capacity");
    if (!elements(d_cn, 3, &cn)) return fail(msg, cap, ORACLE_INVALID, "selective_scan: C element count exceeds int32 capacity");
    if (!elements(d_an, 2, &an)) return fail(msg, cap, ORACLE_INVALID, "selective_scan: A element count exceeds int32 capacity");
    const struct { size_t have, need; const char* name; } sizes[6] = {
        {n_u, ud, "u"}, {n_delta, ud, "delta"}, {n_a, an, "A"}, {n_b, bn, "B"}, {n_c, cn, "C"},
        {n_d, s->has_d ? (size_t)s->channels : 0, "D"}};
    for (int i = 0; i < 6; ++i)
        if (sizes[i].have != sizes[i].need) {
            snprintf(text, sizeof text, "selective_scan: %s has %zu values, shape needs %zu", sizes[i].name, sizes[i].have, sizes[i].need);
            return fail(msg, cap, ORACLE_INVALID, text);
        }
    if (!expect_finite(u, n_u, "u", msg, cap) || !expect_finite(delta, n_delta, "delta", msg, cap) ||
        !expect_finite(a, n_a, "A", msg, cap) || !expect_finite(b, n_b, "B", msg, cap) ||
        !expect_finite(c, n_c, "C", msg, cap) || !expect_finite(d, n_d, "D", msg, cap))
        return ORACLE_INVALID;

    const size_t L = s->length, Dc = s->channels, N = s->state;
    double h[32];
    for (size_t bb = 0; bb < s->batch; ++bb) {
        for (size_t ch = 0; ch < Dc; ++ch) {
            const float* a_row = a + (s->a_rows == 1 ? 0 : ch * N);
            for (size_t n = 0; n < N; ++n) h[n] = 0.0;
            for (size_t t = 0; t < L; ++t) {
                const size_t token = bb * L + t;
                const double uu = u[token * Dc + ch];
                const double dt = sacc_oracle_softplus(delta[token * Dc + ch]);
                double acc = 0.0;
                for (size_t n = 0; n < N; ++n) {
                    const double decay = exp(dt * a_row[n]);
                    if (!in_range(decay, "decay", bb, t, ch, msg, cap)) return ORACLE_RANGE;
                    const double drive = dt * b[token * N + n] * uu;
                    if (!in_range(drive, "drive", bb, t, ch, msg, cap)) return ORACLE_RANGE;
                    h[n] = decay * h[n] + drive;
                    if (!in_range(h[n], "state", bb, t, ch, msg, cap)) return ORACLE_RANGE;
                    const double term = c[token * s->c_width + (s->c_width == 1 ? 0 : n)] * h[n];
                    if (!in_range(term, "C*state", bb, t, ch, msg, cap)) return ORACLE_RANGE;
                    acc += term;
                }
                if (s->has_d) {
                    const double skip = (double)d[ch] * uu;
                    if (!in_range(skip, "D*u", bb, t, ch, msg, cap)) return ORACLE_RANGE;
                    acc += skip;
                }
                if (!in_range(acc, "output", bb, t, ch, msg, cap)) return ORACLE_RANGE;
                y[token * Dc + ch] = acc;
            }
        }
    }
    return ORACLE_OK;
}

/*
 * tests/scan_cuda_suite.hpp:167-204 (scan_bound): first-order running error
 * bound E_y of the reference's FP32 GPU algorithm (docs/SCAN_CUDA.md section 5).
 * A GPU output element passes when |gpu - ref| <= 2 * E_y.  Same layouts as
 * sacc_oracle_scan_ref; inputs are assumed valid.
 */
void sacc_oracle_scan_bound(const OracleShape* s, const float* u, const float* delta, const float* a, const float* b,
                            const float* c, const float* d, double* bound) {
    const double kU = 0x1p-24, kEpsDelta = 6 * kU, kEta = 0x1p-150, kEtaDecay = 0x1p-148;
    int levels = 0;
    while (((size_t)1 << levels) < s->state) ++levels;
    const double g = (levels + 2) * kU / (1 - (levels + 2) * kU);
    const size_t L = s->length, Dc = s->channels, N = s->state;
    double h[32], e[32];
    for (size_t bb = 0; bb < s->batch; ++bb)
        for (size_t ch = 0; ch < Dc; ++ch) {
            const float* a_row = a + (s->a_rows == 1 ? 0 : ch * N);
            for (size_t n = 0; n < N; ++n) h[n] = e[n] = 0.0;
            for (size_t t = 0; t < L; ++t) {
                const size_t token = bb * L + t;
                const double uu = u[token * Dc + ch], dt = sacc_oracle_softplus(delta[token * Dc + ch]);
                double sum_c_e = 0, scale = 0;
                for (size_t n = 0; n < N; ++n) {
                    const double arg = dt * a_row[n], q = exp(arg);
                    const double rho = expm1(fabs(arg) * (kEpsDelta + kU)) * (1 + 4 * kU) + 4 * kU;
                    const double keep = q == 0 ? 0 : q * (1 + rho), lost = q == 0 ? 0 : rho * q;
                    const double r = dt * b[token * N + n] * uu, next = q * h[n] + r;
                    e[n] = ((keep + kEtaDecay) * e[n] + (lost + kEtaDecay) * fabs(h[n]) + (kEpsDelta + 2 * kU) * fabs(r) +
                            kU * fabs(next) + 2 * kEta) / (1 - kU);
                    h[n] = next;
                    const double cv = c[token * s->c_width + (s->c_width == 1 ? 0 : n)];
                    sum_c_e += fabs(cv) * e[n];
                    scale += fabs(cv * next);
                }
                if (s->has_d) scale += fabs((double)d[ch] * uu);
                bound[token * Dc + ch] = (1 + g) * sum_c_e + g * scale + (double)(N + 1) * kEta;
            }
        }
}

/*
 * Extended scan (no counterpart in the reference: the reference contract has
 * zero initial state, no final state, no varlen and no fused gate/bias,
 * include/saccade/selective_scan.hpp:17-18).  The core recurrence is the one
 * of src/selective_scan.cpp:88-107 and reduces to it exactly when every
 * extension is off (tests/test_oracle.py checks that equality bit for bit).
 *
 * layout 0 ("BLD", the reference ABI): u, delta, z, y (batch, length, D);
 *   B (batch, length, groups, N); C (batch, length, groups, c_width).
 * layout 1 ("BDL", Mamba's layout): u, delta, z, y (batch, D, length);
 *   B (batch, groups, N, length); C (batch, groups, c_width, length).
 * Channel d reads group d / (D / groups).
 * delta_bias (D) is added in binary64 before softplus; apply_softplus = 0
 * uses delta as Delta directly (mamba's delta_softplus=False).
 * z (optional) gates the output: y = (sum_n C h + D u) * silu(z).
 * h0 (optional) (nseq, D, N) initial state; h_final (optional) (nseq, D, N).
 * cu_seqlens (optional, nseq + 1 entries, batch must be 1): sequence k is
 *   tokens [cu[k], cu[k+1]) of the length axis, each restarted from h0[k] or 0.
 *   Without cu_seqlens nseq = batch.
 * Inputs are FP32 values (callers round bf16/fp16 inputs to their exact FP32
 * value first); every intermediate is binary64.
 */
typedef struct {
    uint64_t batch, length, channels, state, groups, c_width, a_rows;
    int32_t layout, has_d, has_z, has_bias, apply_softplus, has_h0, want_final, nseq;
} OracleExShape;

/* Element i of an FP32 (f64 == 0) or binary64 (f64 == 1) array, as binary64
 * (FP32 values widen exactly). */
static double rd(const void* p, size_t i, int f64) {
    return f64 ? ((const double*)p)[i] : (double)((const float*)p)[i];
}

/* sigmoid(x) in the reference head's form (src/head_reference.cpp:54-58):
 * 1 / (1 + e^-x) for x >= 0, e^x / (1 + e^x) below. */
static double sigmoid(double x) {
    if (x >= 0) return 1.0 / (1.0 + exp(-x));
    const double e = exp(x);
    return e / (1.0 + e);
}

static void scan_ex_core(const OracleExShape* s, int f64, const void* u, const void* delta, const void* a, const void* b,
                         const void* c, const float* d, const void* z, const float* bias, const float* h0,
                         const int32_t* cu_seqlens, double* y, double* h_final, double* scale) {
    const size_t Bt = s->batch, L = s->length, D = s->channels, N = s->state, G = s->groups, CW = s->c_width;
    const size_t per_group = D / G;
    const size_t nseq = cu_seqlens ? (size_t)s->nseq : Bt;
    double h[64];
    for (size_t seq = 0; seq < nseq; ++seq) {
        const size_t bb = cu_seqlens ? 0 : seq;
        const size_t t0 = cu_seqlens ? (size_t)cu_seqlens[seq] : 0, t1 = cu_seqlens ? (size_t)cu_seqlens[seq + 1] : L;
        for (size_t ch = 0; ch < D; ++ch) {
            const size_t a_row = s->a_rows == 1 ? 0 : ch * N;
            const size_t g = ch / per_group;
            for (size_t n = 0; n < N; ++n) h[n] = s->has_h0 ? (double)h0[(seq * D + ch) * N + n] : 0.0;
            for (size_t t = t0; t < t1; ++t) {
                size_t at, bat0, bstride, cat0, cstride;
                if (s->layout == 0) {
                    at = (bb * L + t) * D + ch;
                    bat0 = ((bb * L + t) * G + g) * N; bstride = 1;
                    cat0 = ((bb * L + t) * G + g) * CW; cstride = 1;
                } else {
                    at = (bb * D + ch) * L + t;
                    bat0 = ((bb * G + g) * N) * L + t; bstride = L;
                    cat0 = ((bb * G + g) * CW) * L + t; cstride = L;
                }
                const double uu = rd(u, at, f64);
                double raw = rd(delta, at, f64);
                if (s->has_bias) raw += (double)bias[ch];
                const double dt = s->apply_softplus ? sacc_oracle_softplus(raw) : raw;
                double acc = 0.0, mag = 0.0;
                for (size_t n = 0; n < N; ++n) {
                    const double decay = exp(dt * rd(a, a_row + n, f64));
                    const double drive = dt * rd(b, bat0 + n * bstride, f64) * uu;
                    h[n] = decay * h[n] + drive;
                    const double term = rd(c, cat0 + (CW == 1 ? 0 : n) * cstride, f64) * h[n];
                    acc += term;
                    mag += fabs(term);
                }
                if (s->has_d) {
                    acc += (double)d[ch] * uu;
                    mag += fabs((double)d[ch] * uu);
                }
                if (s->has_z) {
                    /* y * silu(z), silu(z) = z sigmoid(z) as the reference head's
                     * multiply(y, silu(z)) (src/head_reference.cpp:221 silu, :490 the gate). */
                    const double zz = rd(z, at, f64), gate = zz * sigmoid(zz);
                    acc *= gate;
                    mag *= fabs(gate);
                }
                y[at] = acc;
                /* Term magnitude sum_n |C_n h_n| + |D u| (times |silu(z)|): the
                 * scale that FP32 rounding errors of y grow with. */
                if (scale) scale[at] = mag;
            }
            if (s->want_final)
                for (size_t n = 0; n < N; ++n) h_final[(seq * D + ch) * N + n] = h[n];
        }
    }
}

void sacc_oracle_scan_ex(const OracleExShape* s, const float* u, const float* delta, const float* a, const float* b,
                         const float* c, const float* d, const float* z, const float* bias, const float* h0,
                         const int32_t* cu_seqlens, double* y, double* h_final, double* scale) {
    scan_ex_core(s, 0, u, delta, a, b, c, d, z, bias, h0, cu_seqlens, y, h_final, scale);
}

/* The same scan on binary64 u, delta, A, B, C and z (the activations of the
 * binary64 block oracle, which are not FP32 values); D, the bias and h0 stay
 * FP32 parameters. */
void sacc_oracle_scan_ex_f64(const OracleExShape* s, const double* u, const double* delta, const double* a, const double* b,
                             const double* c, const float* d, const double* z, const float* bias, const float* h0,
                             const int32_t* cu_seqlens, double* y, double* h_final, double* scale) {
    scan_ex_core(s, 1, u, delta, a, b, c, d, z, bias, h0, cu_seqlens, y, h_final, scale);
}

/* silu(x) = x sigmoid(x) elementwise in binary64 with the C library's exp
 * (the reference head's silu value, src/head_reference.cpp:221-232). */
void sacc_oracle_silu(const double* x, size_t n, double* y) {
    for (size_t i = 0; i < n; ++i) y[i] = x[i] * sigmoid(x[i]);
}

/* A = -exp(A_log) in binary64 from FP32 A_log (src/head_reference.cpp:347-354). */
void sacc_oracle_neg_exp(const float* a_log, size_t n, double* a) {
    for (size_t i = 0; i < n; ++i) a[i] = -exp((double)a_log[i]);
}

/* src/selective_scan.cpp:111-116 (cross_scan_source).  Returns (size_t)-1 on a bad argument. */
size_t sacc_oracle_cross_scan_source(size_t direction, size_t token, size_t height, size_t width) {
    if (direction > 3 || height == 0 || width == 0 || token / width >= height) return (size_t)-1;
    const size_t row = token / width, col = token % width;
    const int flip_h = direction == 1 || direction == 3, flip_w = direction == 1 || direction == 2;
    return (flip_h ? height - 1 - row : row) * width + (flip_w ? width - 1 - col : col);
}

/* src/selective_scan.cpp:118-133: x (batch, C, H, W) -> tokens (4 batch, H W, C). */
void sacc_oracle_cross_scan_expand(const float* x, size_t batch, size_t channels, size_t height, size_t width, float* out) {
    const size_t L = height * width;
    for (size_t k = 0; k < 4; ++k)
        for (size_t i = 0; i < batch; ++i)
            for (size_t t = 0; t < L; ++t) {
                const size_t source = sacc_oracle_cross_scan_source(k, t, height, width);
                for (size_t ch = 0; ch < channels; ++ch)
                    out[((k * batch + i) * L + t) * channels + ch] = x[(i * channels + ch) * L + source];
            }
}

/* src/selective_scan.cpp:135-154: tokens -> (batch, C, H, W), mean of the four directions. */
void sacc_oracle_cross_scan_merge(const double* y, size_t batch, size_t channels, size_t height, size_t width, double* out) {
    const size_t L = height * width;
    for (size_t i = 0; i < batch; ++i)
        for (size_t ch = 0; ch < channels; ++ch)
            for (size_t p = 0; p < L; ++p) {
                double sum = 0.0;
                for (size_t k = 0; k < 4; ++k)
                    sum += y[((k * batch + i) * L + sacc_oracle_cross_scan_source(k, p, height, width)) * channels + ch];
                out[(i * channels + ch) * L + p] = sum / 4.0;
            }
}
