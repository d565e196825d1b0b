// mamba_block.cpp -- forward of one Mamba block around the selective scan,
// the layers the reference builds from TensorRT layers around its scan plugin
// (src/head_trt_network.cpp:181-233; binary64 twin
// src/head_reference.cpp:471-495), plus BASELINE's RMSNorm prologue:
//
//   r      = 1 / sqrt(mean(x^2) + eps)                    rms_prep (x once), which also forms
//                                                          W_in diag(w) in the same launch
//   xz     = diag(r) x (W_in diag(w))^T                   one tcgen05 GEMM, row scale epilogue
//   u      = silu(causal_conv1d(x_in) + conv_b)           conv_silu on the x_in half of xz
//   dbc    = u W_x^T = [dt | B | C]                       one tcgen05 GEMM (N = dt_rank + 2 d_state)
//   delta  = dt W_dt^T                                    tcgen05 GEMM on the dt columns of dbc
//   y      = scan(u, delta + dt_bias, A, B, C, D) * silu(z)   bulk scan, (B, L, D), z / B / C read
//                                                          in place from xz and dbc (row pitches)
//   out    = y W_out^T + x                                tcgen05 GEMM, residual epilogue
//
// launch_cross_block runs one Cross-Scan head level (expand, this block with
// the residual on the tokens, merge) with in_proj and out_proj once per map
// position instead of once per direction token (cross_block.cu).
//
// Intermediates live in a caller-provided workspace (sacc_mamba_block_workspace
// gives its size); nothing is allocated.  The batch is split into chunks
// whose (batch, length, d_inner) tensors stay within the scan's int32 element
// capacity.
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "internal.h"

namespace sacc {
namespace {

struct Layout {
    std::size_t r, wn, wx, xz, u, dbc, delta, y, scan, scan_bytes, total;
    bool fuse_dt; // dt_proj inside the scan
};

// Batch rows per scan call: the bulk scan indexes rows (batch x channels) and
// tokens (batch x length) with 32-bit integers and everything else with
// 64-bit ones, so a call may hold any batch whose rows and tokens stay below
// 2^31 (config 4's 512 x 4096 x 2048 layer is one call: 8192 units, 13.8 waves,
// instead of eight 1024-unit calls of two waves, the second 73 % full).
std::uint64_t scan_rows(const SaccMambaBlockArgs& a) {
    std::uint64_t chunk = a.batch;
    while (chunk > 1 && (chunk * a.d_inner > kMaxElements || chunk * a.length > kMaxElements)) chunk = (chunk + 1) / 2;
    return chunk;
}

// dt_proj inside the scan (delta = dt W_dt^T formed per token in FP32, no
// GEMM launch and no delta tensor) for the small ranks the scan supports.
bool dt_rank_fusable(const SaccMambaBlockArgs& a) { return a.dt_rank == 8 || a.dt_rank == 16; }

// The scan's arguments for `nb` rows of the block (pointers left null).
SaccScanExArgs scan_shape(const SaccMambaBlockArgs& a, std::uint64_t nb) {
    SaccScanExArgs s{};
    s.batch = nb; s.length = a.length; s.channels = a.d_inner; s.state = a.d_state; s.groups = 1; s.a_rows = a.d_inner;
    s.c_width = a.d_state; s.layout = SACC_LAYOUT_BLD; s.dtype = a.dtype; s.delta_softplus = 1; s.nseq = 0;
    return s;
}

std::size_t align256(std::size_t v) { return (v + 255) & ~std::size_t(255); }

Layout plan(const SaccMambaBlockArgs& a) {
    const std::size_t e = 2; // bf16 / fp16 activations
    const std::size_t M = a.batch * a.length, D = a.d_inner, N = a.d_state, R = a.dt_rank, dm = a.d_model;
    Layout l{};
    std::size_t off = 0;
    auto take = [&](std::size_t bytes) {
        const std::size_t at = off;
        off = align256(off + bytes);
        return at;
    };
    l.r = take(M * sizeof(float));
    l.wn = take(2 * D * dm * e);
    l.wx = a.c_width == 1 ? take((R + 2 * N) * D * e) : 0; // W_x with its C row repeated d_state times
    l.xz = take(M * 2 * D * e);
    l.u = take(M * D * e);
    l.dbc = take(M * (R + 2 * N) * e);
    // Scratch of the scan's fused chunk-parallel mode (few long sequences);
    // that launch runs without the in-scan dt_proj (its per-token dot product
    // sits on the critical path there: 156 -> 170 us for the three HR levels),
    // every other scan forms delta itself for rank 8 / 16 (HR L = 60, four
    // threads per lane: 46 -> 38 us; config 1: 55 -> 51 us).
    l.scan_bytes = bulk_scan_scratch_bytes(scan_shape(a, a.batch < scan_rows(a) ? a.batch : scan_rows(a)));
    l.fuse_dt = dt_rank_fusable(a) && l.scan_bytes == 0;
    l.delta = l.fuse_dt ? 0 : take(M * D * e);
    l.y = take(M * D * e);
    l.scan = l.scan_bytes ? take(l.scan_bytes) : 0;
    l.total = off;
    return l;
}

SaccGemmArgs gemm_args(int dtype, std::uint64_t m, std::uint64_t n, std::uint64_t k, const void* a, std::uint64_t lda,
                       const void* b, std::uint64_t ldb, void* c, std::uint64_t ldc) {
    SaccGemmArgs g{};
    g.m = m; g.n = n; g.k = k; g.lda = lda; g.ldb = ldb; g.ldc = ldc;
    g.in_dtype = dtype; g.out_dtype = dtype;
    g.a = a; g.b = b; g.c = c;
    return g;
}

// x_proj, dt_proj and the selective scan of a block's batch x length tokens:
// u (M, D); the gate z row t at z + t * zld; wx (a rank-1 C's repeated W_x),
// dbc, delta (unused when fuse_dt), y (M, D) and the scan scratch from the
// caller's workspace.
// The scan scratch's hand-off flags were cleared by the conv kernel before
// (ZeroSpan), so the first scan launch needs no memset; a later batch chunk
// reuses the scratch and clears them itself.
cudaError_t xproj_scan(const SaccMambaBlockArgs& a, const void* u, const void* z, std::uint64_t zld, void* wx, void* dbc,
                       void* delta, void* y, unsigned char* scan, std::size_t scan_bytes, bool fuse_dt, cudaStream_t stream) {
    const std::uint64_t M = a.batch * a.length, D = a.d_inner, N = a.d_state, R = a.dt_rank;
    const std::uint64_t W = R + 2 * N; // dbc row: dt | B | C
    const int dt_ = a.dtype;
    const std::size_t e = 2;
    auto at = [&](const void* p, std::size_t elems) { return static_cast<const unsigned char*>(p) + elems * e; };
    cudaError_t err;
    // x_proj in one GEMM: dt (R), B (N), C (N) as column slices of dbc.  A
    // rank-1 C (one value per token) runs as a full C whose N columns are
    // that value: W_x's C row is repeated N times, so every C column is the
    // same dot product and the scan's sum over C_n h_n is the rank-1 result.
    const void* w_x = a.w_x;
    if (a.c_width == 1) {
        if ((err = launch_repeat_last_row(dt_, a.w_x, R + N + 1, N, D, wx, stream)) != cudaSuccess) return err;
        w_x = wx;
    }
    if ((err = launch_gemm(gemm_args(dt_, M, W, D, u, D, w_x, D, dbc, W), stream)) != cudaSuccess) return err;
    // dt_proj on the dt columns (bias added inside the scan, before softplus);
    // for rank 8 / 16 the scan forms delta itself.
    if (!fuse_dt && (err = launch_gemm(gemm_args(dt_, M, D, R, dbc, W, a.w_dt, R, delta, D), stream)) != cudaSuccess)
        return err;

    // Selective scan with D skip and SiLU(z) gate, (B, L, D) layout, z / B / C
    // read in place through their row pitches; chunked by batch only where
    // the scan's 32-bit row / token indices require it.
    const RowStrides pitch{zld, W, W};
    const std::uint64_t chunk = scan_rows(a);
    for (std::uint64_t b0 = 0; b0 < a.batch; b0 += chunk) {
        const std::uint64_t nb = (a.batch - b0 < chunk) ? a.batch - b0 : chunk;
        const std::size_t tok = b0 * a.length;
        SaccScanExArgs s = scan_shape(a, nb);
        s.u = at(u, tok * D);
        s.delta = fuse_dt ? at(dbc, tok * W) : at(delta, tok * D);
        s.z = at(z, tok * zld);
        s.b = at(dbc, tok * W + R); s.c = at(dbc, tok * W + R + N);
        s.a = a.a; s.d = a.d; s.delta_bias = a.dt_bias;
        s.y = static_cast<unsigned char*>(y) + tok * D * e;
        if (!bulk_eligible(s, &pitch)) return cudaErrorInvalidValue; // shapes are checked by the caller
        const DtFusion dtf{at(dbc, tok * W), W, a.w_dt, static_cast<int>(R)};
        if (fuse_dt && !dt_fusable(s, dtf)) return cudaErrorInvalidValue;
        if ((err = launch_scan_bulk(s, stream, &pitch, scan_bytes ? scan : nullptr, scan_bytes, fuse_dt ? &dtf : nullptr,
                                    b0 == 0)) != cudaSuccess)
            return err;
    }
    return cudaSuccess;
}

// Workspace of one Cross-Scan head level: P = images x positions map rows,
// M = 4 P direction tokens.
struct CrossLayout {
    std::size_t r, wn, wx, rows, xz, u, z, dbc, delta, y, mean, out_rows, scan, scan_bytes, total;
    bool fuse_dt;
};

// The block as the scan sees a level: four sequences (one per direction) of
// height x width tokens per image, sequence k * images + image.
SaccMambaBlockArgs cross_inner(const SaccCrossScanBlockArgs& c) {
    SaccMambaBlockArgs v = c.block;
    v.batch = 4 * c.block.batch;
    v.length = c.height * c.width;
    return v;
}

CrossLayout plan_cross(const SaccCrossScanBlockArgs& c) {
    const SaccMambaBlockArgs v = cross_inner(c);
    const std::size_t e = 2;
    const std::size_t P = c.block.batch * v.length, M = v.batch * v.length;
    const std::size_t D = v.d_inner, N = v.d_state, R = v.dt_rank, dm = v.d_model;
    CrossLayout l{};
    std::size_t off = 0;
    auto take = [&](std::size_t bytes) {
        const std::size_t at = off;
        off = align256(off + bytes);
        return at;
    };
    l.r = take(P * sizeof(float));
    l.wn = take(2 * D * dm * e);
    l.wx = v.c_width == 1 ? take((R + 2 * N) * D * e) : 0;
    l.rows = take(P * dm * e);
    l.xz = take(P * 2 * D * e);
    l.u = take(M * D * e);
    l.z = take(M * D * e);
    l.dbc = take(M * (R + 2 * N) * e);
    l.scan_bytes = bulk_scan_scratch_bytes(scan_shape(v, v.batch < scan_rows(v) ? v.batch : scan_rows(v)));
    l.fuse_dt = dt_rank_fusable(v) && l.scan_bytes == 0;
    l.delta = l.fuse_dt ? 0 : take(M * D * e);
    l.y = take(M * D * e);
    l.mean = take(P * D * e);
    l.out_rows = take(P * dm * sizeof(float));
    l.scan = l.scan_bytes ? take(l.scan_bytes) : 0;
    l.total = off;
    return l;
}

} // namespace

std::size_t mamba_block_workspace(const SaccMambaBlockArgs& a) { return plan(a).total; }

cudaError_t launch_mamba_block(const SaccMambaBlockArgs& a, void* workspace, cudaStream_t stream) {
    const Layout l = plan(a);
    auto* ws = static_cast<unsigned char*>(workspace);
    float* r = reinterpret_cast<float*>(ws + l.r);
    void* wn = ws + l.wn;
    void *xz = ws + l.xz, *u = ws + l.u, *dbc = ws + l.dbc, *delta = ws + l.delta, *y = ws + l.y;
    const std::uint64_t M = a.batch * a.length, D = a.d_inner, dm = a.d_model;
    const int dt_ = a.dtype;
    const std::size_t e = 2;
    auto at = [&](const void* p, std::size_t elems) { return static_cast<const unsigned char*>(p) + elems * e; };
    cudaError_t err;

    // RMSNorm folded into in_proj: per-token scale r, weight columns scaled by w.
    const bool norm = a.norm_w != nullptr;
    const void* w_in = a.w_in;
    if (norm) {
        if ((err = launch_rms_prep(dt_, a.x, M, static_cast<unsigned>(dm), a.eps, r, a.w_in, a.norm_w, 2 * D, wn, stream)) !=
            cudaSuccess)
            return err;
        w_in = wn;
    }
    // in_proj: x_in and z side by side in one (M, 2D) output.
    SaccGemmArgs g = gemm_args(dt_, M, 2 * D, dm, a.x, dm, w_in, dm, xz, 2 * D);
    g.row_scale = norm ? r : nullptr;
    if ((err = launch_gemm(g, stream)) != cudaSuccess) return err;

    // Causal depthwise conv1d (width d_conv) + SiLU on the x_in half.
    if ((err = launch_conv_silu(dt_, static_cast<int>(a.d_conv), xz, 2 * D, a.conv_w, a.conv_b, a.batch, a.length, D, u,
                                stream, bulk_scan_flags(l.scan_bytes ? ws + l.scan : nullptr, l.scan_bytes))) != cudaSuccess)
        return err;

    // x_proj, dt_proj and the scan; the gate z is the second half of each xz row.
    if ((err = xproj_scan(a, u, at(xz, D), 2 * D, ws + l.wx, dbc, delta, y, ws + l.scan, l.scan_bytes, l.fuse_dt, stream)) !=
        cudaSuccess)
        return err;

    // out_proj + residual.
    g = gemm_args(dt_, M, dm, D, y, D, a.w_out, D, a.out, dm);
    g.residual = a.residual ? a.x : nullptr;
    g.ldr = dm;
    return launch_gemm(g, stream);
}

std::size_t cross_block_workspace(const SaccCrossScanBlockArgs& c) { return plan_cross(c).total; }

cudaError_t launch_cross_block(const SaccCrossScanBlockArgs& c, void* workspace, cudaStream_t stream) {
    const CrossLayout l = plan_cross(c);
    const SaccMambaBlockArgs& a = c.block;
    const SaccMambaBlockArgs v = cross_inner(c);
    auto* ws = static_cast<unsigned char*>(workspace);
    float* r = reinterpret_cast<float*>(ws + l.r);
    void *rows = ws + l.rows, *xz = ws + l.xz, *u = ws + l.u, *z = ws + l.z, *mean = ws + l.mean;
    const std::uint64_t B = a.batch, L = v.length, P = B * L, D = a.d_inner, dm = a.d_model;
    const int dt_ = a.dtype;
    cudaError_t err;

    // The maps as position-major rows, then in_proj once per position (with
    // the RMSNorm fold of the block when norm_w is given).
    if ((err = launch_rows_from_maps(dt_, c.x, B, L, dm, rows, stream)) != cudaSuccess) return err;
    const bool norm = a.norm_w != nullptr;
    const void* w_in = a.w_in;
    if (norm) {
        if ((err = launch_rms_prep(dt_, rows, P, static_cast<unsigned>(dm), a.eps, r, a.w_in, a.norm_w, 2 * D, ws + l.wn, stream)) !=
            cudaSuccess)
            return err;
        w_in = ws + l.wn;
    }
    SaccGemmArgs g = gemm_args(dt_, P, 2 * D, dm, rows, dm, w_in, dm, xz, 2 * D);
    g.row_scale = norm ? r : nullptr;
    if ((err = launch_gemm(g, stream)) != cudaSuccess) return err;

    // Every direction's conv + SiLU and gate, read through the flips.
    if ((err = launch_cross_conv(dt_, xz, a.conv_w, a.conv_b, B, c.height, c.width, D, u, z, stream,
                                 bulk_scan_flags(l.scan_bytes ? ws + l.scan : nullptr, l.scan_bytes))) != cudaSuccess)
        return err;
    if ((err = xproj_scan(v, u, z, D, ws + l.wx, ws + l.dbc, ws + l.delta, ws + l.y, ws + l.scan, l.scan_bytes, l.fuse_dt,
                          stream)) != cudaSuccess)
        return err;

    // The merge of the gated outputs per position, out_proj per position
    // (FP32 rows), and the rows back to the maps with x as the residual.
    if ((err = launch_cross_mean(dt_, ws + l.y, B, c.height, c.width, D, mean, stream)) != cudaSuccess) return err;
    float* orows = reinterpret_cast<float*>(ws + l.out_rows);
    g = gemm_args(dt_, P, dm, D, mean, D, a.w_out, D, orows, dm);
    g.out_dtype = SACC_DTYPE_F32;
    if ((err = launch_gemm(g, stream)) != cudaSuccess) return err;
    if ((err = launch_maps_from_rows(orows, a.residual ? c.x : nullptr, B, L, dm, c.out, stream)) != cudaSuccess) return err;
    return cudaSuccess;
}

} // namespace sacc
