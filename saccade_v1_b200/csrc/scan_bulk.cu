// scan_bulk.cu -- high-throughput selective scan for 16-bit activations with
// FP32 state and N = 16 states, in Mamba's (B, D, L)
// layout or the reference's (B, L, D) layout.
//
// Work split: one thread owns one (batch, channel) lane and its 16 states in
// registers; a CTA of 128 threads owns 128 consecutive channels of one batch
// row and walks the sequence in chunks of 32 tokens.
//
// Data movement: per chunk, one thread issues TMA loads of the u / delta / z
// tiles and of the B / C tiles into a two-stage ring completed by mbarriers,
// and a TMA store of the y tile, which the outputs share with the consumed u
// tile of the stage.  In (B, D, L) each thread's 32 tokens are one
// 64-byte row of a 64-byte-swizzled tile, read with conflict-free 16-byte
// shared loads; in (B, L, D) a warp reads 32 consecutive channels of one
// token.  B and C are converted once per chunk to an FP32 token-major table
// that all threads read with broadcast loads.  Every input byte crosses HBM
// once, every output byte once.
//
// Arithmetic: with N = 16 the scan is bound by its arithmetic, not by HBM.
// Every state update needs its decay exp(Delta A[n]) and three FP32
// operations (Delta u B, the state FMA and the C h FMA) against 6 bytes of
// bf16 traffic per 16 updates.  For S4D-real A (A[n] = (n + 1) A[0]) the 16
// decays of a token are powers of one exponential, a product tree of packed
// multiplies (scan_block8_pow), and the FP32 FMA pipe binds; for any other A
// each decay is one 2^x on the special-function unit, which binds.  softplus
// runs on the FMA pipe except for one ex2 (log1p(e) = e * P(e), a degree-5
// minimax fit with 8.5e-6 relative error, gen_softplus_poly.py).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstring>
#include <random>
#include <mutex>
#include <string>
#include <type_traits>

#include "internal.h"
#include "scan_common.cuh"
#include "tma.cuh"

namespace sacc {

__device__ unsigned int g_bulk_fault; // set when a bounded wait ran out; read by sacc_scan_fault()

namespace {

constexpr int kLanes = 128; // threads (lanes) per CTA
constexpr int kT = 32;      // tokens per chunk
constexpr int kStages = 2;
constexpr int kN = 16;
#ifndef SACC_BULK_MIN5
#define SACC_BULK_MIN5 1
#endif
// CTAs per SM the register budget is set for: five (96 registers a thread)
// for the multi-wave walk of the split launch (kMode 1), where the SMs stay
// full; four (128) for one-wave launches (a CTA gets more of its SM), the
// fused chunk-parallel mode, the in-scan delta and a staged gate tile.
constexpr int bulk_min_blocks(int mode, int rank, bool ztile) {
    return (SACC_BULK_MIN5 && mode == 1 && rank == 0 && !ztile) ? 5 : 4;
}
constexpr int kMaxFusedParts = 32;

// How the gate reaches shared memory (see Smem): 0 not at all (no gate, or
// the scan forms delta itself and reads the gate from global memory), 1 a
// tile per stage (the fused chunk-parallel walk), 2 one chunk's tile as two
// 16-token halves (one-item walks: four CTAs per SM instead of three).
__host__ __device__ constexpr int gate_mode(bool has_z, int rank, bool bdl, int mode) {
    return !has_z || rank != 0 ? 0 : (mode != 2 ? 2 : 1);
}

// One item of work: 128 channels of one row (or packed sequence) over the
// chunk range of one part, with the tensor-map coordinates of the unit.
struct Item {
    unsigned long long b, d0, tok0, len;
    int c0, c1, part, pass, row0, bb, brow0, crow0;
    int last; // the range ends the row (c1 is the row's chunk count)
};

// The producer's position in a CTA's list of (item, chunk) loads.
struct Cursor {
    Item w;
    unsigned long long it;
    int chunk, more;
};

// kZ (gate_mode): the gate z staged by TMA, in either layout.  Read from
// global memory instead, (B, L, D) lane by lane, the gated scan was 36 %
// slower than ungated (the loads' latency and 64-bit address arithmetic on
// the FMA pipe; prefetched one token block ahead, slower still).  A gate tile
// per stage (kZ == 1, the fused chunk-parallel walk) holds three CTAs per SM;
// one chunk's tile as two 16-token halves with a barrier each (kZ == 2, the
// one-item walks) holds four: each half of the next chunk's gate loads once
// the current chunk is past that half.  The scan that forms delta itself
// (kR > 0: the block pipeline's short sequences) reads the gate from global
// memory.
// The one-thread-per-lane kernel writes a chunk's outputs over its
// u tile (each thread reads its eight u values of a token block before it
// writes their eight outputs to the same places, and the y tile has the u
// tile's layout), so the stage is free again once the y store has read it.
template <typename T, int kZ>
struct Smem {
    alignas(1024) T u[kStages][kLanes * kT];
    alignas(1024) T dl[kStages][kLanes * kT];
    alignas(1024) T z[kZ == 1 ? kStages : (kZ == 2 ? 2 : 1)][kZ == 1 ? kLanes * kT : (kZ == 2 ? kLanes * kT / 2 : 8)];
    alignas(8) std::uint64_t zfull[kZ == 2 ? 2 : 1]; // kZ == 2: one barrier per half
    alignas(128) T braw[kStages][kN * kT];
    alignas(128) T craw[kStages][kN * kT];
    alignas(16) float bc[kT][2 * kN]; // per token: B[0..15], C[16..31] (C[16] only when rank 1)
    alignas(8) std::uint64_t full[kStages];
    Cursor next; // thread 0 only
};

// The four-threads-per-lane kernel shares a lane's u values among its four
// threads, so its outputs go to a tile of their own.
template <typename T>
struct SmemY : Smem<T, 0> {
    alignas(1024) T y[kLanes * kT];
};

template <typename S>
constexpr size_t smem_bytes() {
    return sizeof(S) + 1024; // + alignment slack for the 1024-byte swizzle atoms
}

struct BulkParams {
    const float *a, *d, *bias, *h0;
    float* h_final;
    const int32_t* cu; // packed varlen sequences ((B, L, D) with batch 1), else null
    void* y;           // plain stores of a varlen sequence's last, partial chunk
    const void* zg;    // (B, L, D) gate, read from global memory
    unsigned long long zld; // its row pitch (elements between tokens)
    unsigned long long length, channels, per_group;
    unsigned long long units;    // (rows or packed sequences) x 128-channel tiles
    unsigned long long epoch;    // this launch's hand-off flag value (split launches)
    unsigned groups;
    int a_shared, c_full, has_d, softplus, nchunks;
    int parts;                   // chunk ranges per unit (> 1: split launch, chunk-parallel phases or the fused launch)
    int phase;                   // 0 one pass; chunk-parallel: 1 local pass (parts from zero), 2 final pass
    int passes;                  // 2: fused chunk-parallel launch (pass 0 local, pass 1 final, one CTA per part)
    unsigned long long item0;    // first item of this launch (the final pass starts at part 1)
    float* scratch;              // fused mode: per (unit, part) 17 x 128 floats (S, sum of Delta), then the flags
    const void* wdt;             // kR > 0: W_dt (channels x kR); delta = dt rows (tensor map td) x W_dt^T in the scan
};


template <typename T>
__device__ __forceinline__ float2 unpack2(std::uint32_t w);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(std::uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(std::uint32_t w) {
    __half2 h;
    std::memcpy(&h, &w, 4);
    return __half22float2(h);
}

template <typename T>
__device__ __forceinline__ std::uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ std::uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    std::uint32_t w;
    std::memcpy(&w, &v, 4);
    return w;
}
template <>
__device__ __forceinline__ std::uint32_t pack2<__half>(float lo, float hi) {
    const __half2 v = __floats2half2_rn(lo, hi);
    std::uint32_t w;
    std::memcpy(&w, &v, 4);
    return w;
}

// A lane's 16 FP32 values (a row of A, h0 or h_final) as four 16-byte accesses
// (rows are 64-byte aligned: the launcher checks the base pointers).
__device__ __forceinline__ void load16(const float* src, float (&v)[16], float scale = 1.0f) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float4 q = __ldg(reinterpret_cast<const float4*>(src) + k);
        v[4 * k] = q.x * scale; v[4 * k + 1] = q.y * scale; v[4 * k + 2] = q.z * scale; v[4 * k + 3] = q.w * scale;
    }
}

__device__ __forceinline__ void store16(float* dst, const float (&v)[16]) {
#pragma unroll
    for (int k = 0; k < 4; ++k)
        reinterpret_cast<float4*>(dst)[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
}

// Eight tokens of one lane's u / raw delta / z.
struct Block8 {
    float u[8], x[8], z[8];
};

// (B, D, L): row `tid` of a 64-byte-swizzled [128][32] tile; chunk q of row r
// sits at q ^ ((r >> 1) & 3) (TMA 64-byte swizzle: address bits [4:5] ^= [7:8]).
// kZHalves: the gate from the two-half tile, each half [128 rows][16 tokens]
// without swizzle (one 16-byte read per token block).
template <typename T, bool kHasZ, bool kZHalves = false>
__device__ __forceinline__ void load_block_bdl(const T* u, const T* dl, const T* z, int tid, int q, Block8& blk) {
    const int off = tid * kT + ((q ^ ((tid >> 1) & 3)) << 3);
    const uint4 uq = *reinterpret_cast<const uint4*>(u + off);
    const uint4 xq = *reinterpret_cast<const uint4*>(dl + off);
    const std::uint32_t uw[4] = {uq.x, uq.y, uq.z, uq.w}, xw[4] = {xq.x, xq.y, xq.z, xq.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 a = unpack2<T>(uw[j]), b = unpack2<T>(xw[j]);
        blk.u[2 * j] = a.x; blk.u[2 * j + 1] = a.y;
        blk.x[2 * j] = b.x; blk.x[2 * j + 1] = b.y;
    }
    if constexpr (kHasZ) {
        const uint4 zq = *reinterpret_cast<const uint4*>(
            kZHalves ? z + (q >> 1) * (kLanes * kT / 2) + tid * (kT / 2) + ((q & 1) << 3) : z + off);
        const std::uint32_t zw[4] = {zq.x, zq.y, zq.z, zq.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 c = unpack2<T>(zw[j]);
            blk.z[2 * j] = c.x; blk.z[2 * j + 1] = c.y;
        }
    }
}

template <typename T>
__device__ __forceinline__ void store_block_bdl(T* y, int tid, int q, const float (&out)[8]) {
    const int off = tid * kT + ((q ^ ((tid >> 1) & 3)) << 3);
    *reinterpret_cast<uint4*>(y + off) = make_uint4(pack2<T>(out[0], out[1]), pack2<T>(out[2], out[3]),
                                                    pack2<T>(out[4], out[5]), pack2<T>(out[6], out[7]));
}

// (B, L, D): token-major [32][128] tiles; lane `tid` is column tid.  With
// kZTile the gate comes from its own tile (tokens past a tensor's end read as
// zero), else the first `count` tokens' gate from global memory (token rows
// zrow0 + ..., pitch zld).
template <typename T, bool kHasZ, bool kZTile>
__device__ __forceinline__ void load_block_bld(const T* u, const T* dl, const T* z, const T* zg, unsigned long long zrow0,
                                               unsigned long long zld, unsigned long long d, int tid, int q, int count,
                                               Block8& blk) {
    if constexpr (kHasZ && !kZTile) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
            blk.z[j] = j < count ? to_f32(zg[(zrow0 + static_cast<unsigned long long>(q * 8 + j)) * zld + d]) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int at = (q * 8 + j) * kLanes + tid;
        blk.u[j] = to_f32(u[at]);
        blk.x[j] = to_f32(dl[at]);
        if constexpr (kHasZ && kZTile) blk.z[j] = to_f32(z[at]);
    }
}

// (B, L, D) with delta formed in the scan: the chunk's dt rows sit token-major
// in `dt` ([32][kR]); delta of token t is dt[t] . W_dt[d] (FP32; `wrow` the
// lane's W_dt row, re-read from L1 for every 8 tokens so that it holds no
// registers across the scan).  Every lane reads the same dt values (broadcast).
template <typename T, int kR>
__device__ __forceinline__ void delta_from_dt(const T* dt, const T* wrow, int q, Block8& blk) {
    float wd[kR];
#pragma unroll
    for (int v = 0; v < kR / 8; ++v) {
        const uint4 w8 = __ldg(reinterpret_cast<const uint4*>(wrow) + v);
        const std::uint32_t ww[4] = {w8.x, w8.y, w8.z, w8.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = unpack2<T>(ww[i]);
            wd[8 * v + 2 * i] = f.x;
            wd[8 * v + 2 * i + 1] = f.y;
        }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint4* row = reinterpret_cast<const uint4*>(dt + (q * 8 + j) * kR);
        float acc = 0.0f;
#pragma unroll
        for (int v = 0; v < kR / 8; ++v) {
            const uint4 w8 = row[v];
            const std::uint32_t ww[4] = {w8.x, w8.y, w8.z, w8.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = unpack2<T>(ww[i]);
                acc = fmaf(f.x, wd[8 * v + 2 * i], acc);
                acc = fmaf(f.y, wd[8 * v + 2 * i + 1], acc);
            }
        }
        blk.x[j] = acc;
    }
}

template <typename T>
__device__ __forceinline__ void store_block_bld(T* y, int tid, int q, const float (&out)[8]) {
#pragma unroll
    for (int j = 0; j < 8; ++j) y[(q * 8 + j) * kLanes + tid] = from_f32<T>(out[j]);
}

// Loads of the chunk starting at token t0 into stage s.  (B, D, L): 2D maps,
// x = token, y = row (b * D + d).  (B, L, D): 3D maps (channel, token, batch),
// so that a chunk past the end of a sequence reads zeros instead of the next
// sequence; a packed varlen sequence reads whatever follows it, unused.
// kZ == 1: the gate's tile is staged with the others (in (B, L, D) as two
// 16-token boxes); kZ == 2 stages it apart (issue_gate_half); the four-thread
// kernel reads the gate from global memory.
template <typename T, bool kBDL, bool kHasZ, int kR = 0, int kZ = 0>
__device__ __forceinline__ void issue_chunk(Smem<T, kZ>& sm, int s, int t0, int row0, int brow0, int crow0, int bb,
                                            std::uint32_t c_bytes, const CUtensorMap* tu, const CUtensorMap* td,
                                            const CUtensorMap* tz, const CUtensorMap* tb, const CUtensorMap* tc) {
    constexpr bool kZTile = kZ == 1;
    static_assert(!kZ || kHasZ, "a gate tile needs a gate");
    constexpr std::uint32_t tile = kLanes * kT * sizeof(T), btile = kN * kT * sizeof(T);
    if constexpr (kR > 0) {
        // (B, L, D), delta formed in the scan: the chunk's dt rows instead of a delta tile.
        mbar_arrive_expect_tx(&sm.full[s], tile * (kZTile ? 2u : 1u) + kR * kT * sizeof(T) + btile + c_bytes);
        tma_load_3d(sm.u[s], tu, &sm.full[s], row0, t0, bb);
        tma_load_3d(sm.dl[s], td, &sm.full[s], 0, t0, bb);
        if constexpr (kZTile) {
            tma_load_3d(sm.z[s], tz, &sm.full[s], row0, t0, bb);
            tma_load_3d(sm.z[s] + kLanes * kT / 2, tz, &sm.full[s], row0, t0 + kT / 2, bb);
        }
        tma_load_3d(sm.braw[s], tb, &sm.full[s], brow0, t0, bb);
        tma_load_3d(sm.craw[s], tc, &sm.full[s], crow0, t0, bb);
        return;
    }
    mbar_arrive_expect_tx(&sm.full[s], tile * (kZTile ? 3u : 2u) + btile + c_bytes);
    if (kBDL) {
        tma_load_2d(sm.u[s], tu, &sm.full[s], t0, row0);
        tma_load_2d(sm.dl[s], td, &sm.full[s], t0, row0);
        if constexpr (kZTile) tma_load_2d(sm.z[s], tz, &sm.full[s], t0, row0);
        tma_load_2d(sm.braw[s], tb, &sm.full[s], t0, brow0);
        tma_load_2d(sm.craw[s], tc, &sm.full[s], t0, crow0);
    } else {
        tma_load_3d(sm.u[s], tu, &sm.full[s], row0, t0, bb);
        tma_load_3d(sm.dl[s], td, &sm.full[s], row0, t0, bb);
        if constexpr (kZTile) {
            tma_load_3d(sm.z[s], tz, &sm.full[s], row0, t0, bb);
            tma_load_3d(sm.z[s] + kLanes * kT / 2, tz, &sm.full[s], row0, t0 + kT / 2, bb);
        }
        tma_load_3d(sm.braw[s], tb, &sm.full[s], brow0, t0, bb);
        tma_load_3d(sm.craw[s], tc, &sm.full[s], crow0, t0, bb);
    }
}

// kZ == 2: half h (tokens 16 h .. 16 h + 15) of the gate of the chunk at
// token t0 into its half of the single gate tile ((B, D, L): a 16 x 128 box of
// the unswizzled half-box map).
template <typename T, bool kBDL>
__device__ __forceinline__ void issue_gate_half(Smem<T, 2>& sm, int h, int t0, int row0, int bb, const CUtensorMap* tz) {
    mbar_arrive_expect_tx(&sm.zfull[h], kLanes * (kT / 2) * sizeof(T));
    if constexpr (kBDL) tma_load_2d(sm.z[h], tz, &sm.zfull[h], t0 + h * (kT / 2), row0);
    else tma_load_3d(sm.z[h], tz, &sm.zfull[h], row0, t0 + h * (kT / 2), bb);
}

// Eight tokens of one lane through the recurrence; with kGuard only the first
// `count` (fewer in a sequence's last, partial block; the others are left out
// of the state).  With kSum the block's Deltas are added to `dtsum` (the
// chunk-parallel local pass needs them; the split launch's variant, issue
// bound, leaves the add out).
template <bool kFullC, bool kHasZ, bool kGuard, bool kSum>
__device__ __forceinline__ void scan_block8(const float (*bc)[2 * kN], int q, int count, const Block8& blk, const float (&a)[kN],
                                            float (&h)[kN], float bias, float dskip, int softplus, float (&out)[8],
                                            float& dtsum) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        out[j] = 0.0f;
        if (kGuard && j >= count) continue;
        const int t = q * 8 + j;
        const float xv = blk.x[j] + bias;
        const float dt = softplus ? softplus_poly(xv) : xv;
        if constexpr (kSum) dtsum += dt;
        const float du = dt * blk.u[j];
        const float4* bcv = reinterpret_cast<const float4*>(bc[t]);
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const float cr = kFullC ? 0.0f : bc[t][kN];
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
            const float4 bq = bcv[k4];
            const float bb[4] = {bq.x, bq.y, bq.z, bq.w};
            float cc[4] = {cr, cr, cr, cr};
            if constexpr (kFullC) {
                const float4 cq = bcv[4 + k4];
                cc[0] = cq.x; cc[1] = cq.y; cc[2] = cq.z; cc[3] = cq.w;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int n = 4 * k4 + i;
                const float decay = fast_exp2(dt * a[n]);
                h[n] = fmaf(decay, h[n], du * bb[i]);
                acc[i] = fmaf(cc[i], h[n], acc[i]);
            }
        }
        float y = fmaf(dskip, blk.u[j], (acc[0] + acc[1]) + (acc[2] + acc[3]));
        if constexpr (kHasZ) y *= silu(blk.z[j]);
        out[j] = y;
    }
}

// True when this lane's A row is S4D-real in exact FP32 arithmetic:
// A[n] == (n + 1) * A[0] for every n (the S4D-real initialisation
// A[d, n] = -(n + 1) and any per-lane scale of it).  Then
// exp(Delta A[n]) = q^(n + 1) with q = exp(Delta A[0]) exactly in real
// arithmetic, and the decays need one exponential per token instead of 16.
__device__ __forceinline__ bool s4d_row(const float* arow) {
    float v[kN];
    load16(arow, v);
    bool ok = true;
#pragma unroll
    for (int n = 1; n < kN; ++n) ok = ok && v[n] == static_cast<float>(n + 1) * v[0];
    return ok;
}

// scan_block8 for S4D-real rows: q = 2^(Delta a0) from the special-function
// unit once per token, the 16 decays q^1..q^16 by a product tree of packed
// FP32 multiplies (q2 = q q; (q3, q4) = q2 (q1, q2); (q5..q8) = q4 (q1..q4);
// (q9..q16) = q8 (q1..q8): depth 4, each power within a few ulp plus 16 times
// q's own error), and the state and output updates as packed pairs
// (fma.rn.f32x2 / mul.rn.f32x2: half the issue slots of scalar FP32).
// Per token: 2 special-function ops (softplus and q) instead of 17.
template <bool kFullC, bool kHasZ, bool kGuard, bool kSum>
__device__ __forceinline__ void scan_block8_pow(const float (*bc)[2 * kN], int q, int count, const Block8& blk, float a0,
                                                float (&h)[kN], float bias, float dskip, int softplus, float (&out)[8],
                                                float& dtsum) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        out[j] = 0.0f;
        if (kGuard && j >= count) continue;
        const int t = q * 8 + j;
        const float xv = blk.x[j] + bias;
        const float dt = softplus ? softplus_poly(xv) : xv;
        if constexpr (kSum) dtsum += dt;
        const float du = dt * blk.u[j];
        const float q1 = fast_exp2(dt * a0);
        float2 pw[kN / 2];
        pw[0] = make_float2(q1, q1 * q1);
        pw[1] = __fmul2_rn(make_float2(pw[0].y, pw[0].y), pw[0]);
        const float2 q4 = make_float2(pw[1].y, pw[1].y);
        pw[2] = __fmul2_rn(q4, pw[0]);
        pw[3] = __fmul2_rn(q4, pw[1]);
        const float2 q8 = make_float2(pw[3].y, pw[3].y);
#pragma unroll
        for (int k = 0; k < 4; ++k) pw[4 + k] = __fmul2_rn(q8, pw[k]);
        const float2 du2 = make_float2(du, du);
        const float4* bcv = reinterpret_cast<const float4*>(bc[t]);
        const float cr = kFullC ? 0.0f : bc[t][kN];
        float2 acc0 = make_float2(0.0f, 0.0f), acc1 = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
            const float4 bq = bcv[k4];
            float4 cq = make_float4(cr, cr, cr, cr);
            if constexpr (kFullC) cq = bcv[4 + k4];
            const int n = 4 * k4;
            float2 h0 = make_float2(h[n], h[n + 1]), h1 = make_float2(h[n + 2], h[n + 3]);
            h0 = __ffma2_rn(pw[2 * k4], h0, __fmul2_rn(du2, make_float2(bq.x, bq.y)));
            h1 = __ffma2_rn(pw[2 * k4 + 1], h1, __fmul2_rn(du2, make_float2(bq.z, bq.w)));
            acc0 = __ffma2_rn(make_float2(cq.x, cq.y), h0, acc0);
            acc1 = __ffma2_rn(make_float2(cq.z, cq.w), h1, acc1);
            h[n] = h0.x; h[n + 1] = h0.y; h[n + 2] = h1.x; h[n + 3] = h1.y;
        }
        float y = fmaf(dskip, blk.u[j], (acc0.x + acc1.x) + (acc0.y + acc1.y));
        if constexpr (kHasZ) y *= silu(blk.z[j]);
        out[j] = y;
    }
}

template <bool kBDL, bool kFullC>
__device__ __forceinline__ Item item_at(const BulkParams& p, unsigned long long it) {
    Item w;
    // 32-bit index arithmetic: the launcher keeps items, units and channels
    // below 2^31 (64-bit divisions would sit on every CTA's start-up path).
    const unsigned long long D = p.channels, L = p.length;
    const unsigned tiles = static_cast<unsigned>(D / kLanes), units = static_cast<unsigned>(p.units);
    unsigned it32 = static_cast<unsigned>(it);
    w.pass = 0;
    if (p.passes > 1) {
        const unsigned per_pass = units * static_cast<unsigned>(p.parts);
        w.pass = static_cast<int>(it32 / per_pass);
        it32 %= per_pass;
    }
    const unsigned u = it32 % units;
    w.part = static_cast<int>(it32 / units);
    w.b = u / tiles;
    w.d0 = static_cast<unsigned long long>(u % tiles) * kLanes;
    const unsigned long long g = static_cast<unsigned>(w.d0) / static_cast<unsigned>(p.per_group);
    const int cw = kFullC ? kN : 1;
    // Token range: the whole row, or packed sequence b ((B, L, D), batch 1),
    // its cu_seqlens entries clamped to [0, L] so no access leaves the tensors.
    w.tok0 = 0;
    w.len = L;
    if (!kBDL && p.cu) {
        const long long lo = p.cu[w.b], hi = p.cu[w.b + 1];
        w.tok0 = lo < 0 ? 0 : (static_cast<unsigned long long>(lo) > L ? L : static_cast<unsigned long long>(lo));
        const unsigned long long end = hi < 0 ? 0 : (static_cast<unsigned long long>(hi) > L ? L : static_cast<unsigned long long>(hi));
        w.len = end > w.tok0 ? end - w.tok0 : 0;
    }
    const int nch = (!kBDL && p.cu) ? static_cast<int>((w.len + kT - 1) / kT) : p.nchunks;
    w.c0 = p.parts == 1 ? 0 : static_cast<int>(static_cast<unsigned>(w.part * nch) / static_cast<unsigned>(p.parts));
    w.c1 = p.parts == 1 ? nch : static_cast<int>(static_cast<unsigned>((w.part + 1) * nch) / static_cast<unsigned>(p.parts));
    w.last = w.c1 == nch;
    // Fused mode: part 0's local pass is final (no second pass), the last
    // part's local pass is not needed (no part after it).
    if (p.passes > 1 && (w.pass == 1 ? w.part == 0 : w.part + 1 == p.parts)) w.c1 = w.c0;
    w.row0 = kBDL ? static_cast<int>(w.b * D + w.d0) : static_cast<int>(w.d0);
    w.bb = (!kBDL && p.cu) ? 0 : static_cast<int>(w.b);
    w.brow0 = kBDL ? static_cast<int>((w.b * p.groups + g) * kN) : static_cast<int>(g * kN);
    w.crow0 = kBDL ? static_cast<int>((w.b * p.groups + g) * cw) : static_cast<int>(g * cw);
    return w;
}

// Items of a launch: (unit, part) pairs, per pass.
__device__ __forceinline__ unsigned long long item_count(const BulkParams& p) {
    return p.units * static_cast<unsigned long long>(p.parts) * p.passes;
}

// Moves the producer to the next (item, chunk) of this CTA's list, skipping
// items without chunks; `more` drops to 0 past the last one.
template <bool kBDL, bool kFullC>
__device__ __forceinline__ void cursor_next(Cursor& c, const BulkParams& p) {
    if (++c.chunk < c.w.c1) return;
    const unsigned long long items = item_count(p);
    for (c.it += gridDim.x; c.it < items; c.it += gridDim.x) {
        c.w = item_at<kBDL, kFullC>(p, c.it);
        if (c.w.c1 > c.w.c0) {
            c.chunk = c.w.c0;
            return;
        }
    }
    c.more = 0;
}

// Hand-off of a lane's 16 FP32 states from one piece of a split unit to the
// next, through the lane's own first 32 outputs of the next part (not yet
// written: that part's CTA reads them before it stores its outputs there),
// and a 64-bit flag = this launch's epoch in outputs 32..35 of the CTA's first
// lane ((B, D, L)) or in channels 0..3 of token 32 ((B, L, D)).
template <typename T, bool kBDL>
__device__ __forceinline__ T* stash_at(const BulkParams& p, const Item& w, unsigned long long d, unsigned long long tp) {
    T* y = static_cast<T*>(p.y);
    return kBDL ? y + (w.b * p.channels + d) * p.length + tp : y + (w.b * p.length + tp) * p.channels + d;
}

// 16 states (and, for the chunk-parallel local pass, a 17th value: the
// part's sum of Delta) at tokens tp .. tp + 33 of the lane's outputs.
template <typename T, bool kBDL>
__device__ __forceinline__ void stash_put(const BulkParams& p, T* at, const float (&h)[kN], const float* extra) {
    if (kBDL) {
        uint4* q = reinterpret_cast<uint4*>(at);
#pragma unroll
        for (int k = 0; k < 4; ++k)
            q[k] = make_uint4(__float_as_uint(h[4 * k]), __float_as_uint(h[4 * k + 1]), __float_as_uint(h[4 * k + 2]),
                              __float_as_uint(h[4 * k + 3]));
        if (extra) *reinterpret_cast<float*>(at + 2 * kN) = *extra;
    } else {
        std::uint16_t* q = reinterpret_cast<std::uint16_t*>(at);
#pragma unroll
        for (int k = 0; k < kN; ++k) {
            const std::uint32_t v = __float_as_uint(h[k]);
            q[(2 * k) * p.channels] = static_cast<std::uint16_t>(v & 0xffffu);
            q[(2 * k + 1) * p.channels] = static_cast<std::uint16_t>(v >> 16);
        }
        if (extra) {
            const std::uint32_t v = __float_as_uint(*extra);
            q[(2 * kN) * p.channels] = static_cast<std::uint16_t>(v & 0xffffu);
            q[(2 * kN + 1) * p.channels] = static_cast<std::uint16_t>(v >> 16);
        }
    }
}

template <typename T, bool kBDL>
__device__ __forceinline__ void stash_store(const BulkParams& p, const Item& w, unsigned long long d, const float (&h)[kN]) {
    stash_put<T, kBDL>(p, stash_at<T, kBDL>(p, w, d, static_cast<unsigned long long>(w.c1) * kT), h, nullptr);
}

template <typename T, bool kBDL>
__device__ __forceinline__ void stash_store(const BulkParams& p, const Item& w, unsigned long long d, const float (&h)[kN],
                                            float extra) {
    stash_put<T, kBDL>(p, stash_at<T, kBDL>(p, w, d, static_cast<unsigned long long>(w.c1) * kT), h, &extra);
}

// The 17th stashed value (sum of Delta) at the start of `w`'s part.
template <typename T, bool kBDL>
__device__ __forceinline__ float stash_extra(const BulkParams& p, const Item& w, unsigned long long d) {
    const T* at = stash_at<T, kBDL>(p, w, d, static_cast<unsigned long long>(w.c0) * kT);
    if (kBDL) return __ldcg(reinterpret_cast<const float*>(at + 2 * kN));
    const unsigned short* q = reinterpret_cast<const unsigned short*>(at);
    const std::uint32_t lo = __ldcg(q + (2 * kN) * p.channels), hi = __ldcg(q + (2 * kN + 1) * p.channels);
    return __uint_as_float(lo | (hi << 16));
}

template <typename T, bool kBDL>
__device__ __forceinline__ void stash_load(const BulkParams& p, const Item& w, unsigned long long d, float (&h)[kN]) {
    const T* at = stash_at<T, kBDL>(p, w, d, static_cast<unsigned long long>(w.c0) * kT);
    if (kBDL) {
        const uint4* q = reinterpret_cast<const uint4*>(at);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint4 v = __ldcg(q + k);
            h[4 * k] = __uint_as_float(v.x); h[4 * k + 1] = __uint_as_float(v.y);
            h[4 * k + 2] = __uint_as_float(v.z); h[4 * k + 3] = __uint_as_float(v.w);
        }
    } else {
        const unsigned short* q = reinterpret_cast<const unsigned short*>(at);
#pragma unroll
        for (int k = 0; k < kN; ++k) {
            const std::uint32_t lo = __ldcg(q + (2 * k) * p.channels), hi = __ldcg(q + (2 * k + 1) * p.channels);
            h[k] = __uint_as_float(lo | (hi << 16));
        }
    }
}

template <typename T, bool kBDL>
__device__ __forceinline__ unsigned long long* flag_at(const BulkParams& p, const Item& w, unsigned long long tp) {
    T* at = stash_at<T, kBDL>(p, w, w.d0, tp + (kBDL ? 32 : 32));
    return reinterpret_cast<unsigned long long*>(at);
}

__device__ __forceinline__ void flag_release(unsigned long long* f, unsigned long long v) {
    asm volatile("st.release.gpu.global.b64 [%0], %1;" ::"l"(f), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long flag_acquire(const unsigned long long* f) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(f) : "memory");
    return v;
}

// Fused chunk-parallel mode (scratch): flag of part k of w's unit, after the
// units x parts x 17 x 128 floats of the (state, sum of Delta) records.
__device__ __forceinline__ unsigned long long* fused_flag(const BulkParams& p, const Item& w, int k) {
    const unsigned long long unit = w.b * (p.channels / kLanes) + w.d0 / kLanes;
    unsigned long long* flags = reinterpret_cast<unsigned long long*>(p.scratch + p.units * p.parts * (kN + 1) * kLanes);
    return flags + unit * p.parts + k;
}

// The true initial state of part w.part >= 1 from the local records of parts
// 0 .. part - 1: H_1 = S_0, H_{j+1} = exp2(a sum Delta_j) H_j + S_j (the
// recurrence is linear in h, and a part's per-token decays multiply to one
// exponential of the summed exponents).  Thread j < part first waits (bounded)
// for part j's flag; false when a wait ran out.  Records are loaded two
// parts at a time.
__device__ __forceinline__ bool fused_prefix(const BulkParams& p, const Item& w, int tid, const float (&a)[kN], float (&h)[kN]) {
    bool ready = true;
    if (tid < w.part) {
        const unsigned long long* f = fused_flag(p, w, tid);
        ready = false;
        for (std::uint32_t i = 0; i < (1u << 24); ++i) {
            if (flag_acquire(f) == p.epoch) {
                ready = true;
                break;
            }
            __nanosleep(64);
        }
    }
    if (!__syncthreads_and(ready)) return false;
    const unsigned long long unit = w.b * (p.channels / kLanes) + w.d0 / kLanes;
    const float* rec = p.scratch + unit * p.parts * (kN + 1) * kLanes + tid;
#pragma unroll
    for (int n = 0; n < kN; ++n) h[n] = __ldcg(rec + n * kLanes); // S_0: part 0 ran from h0
    constexpr int kBatch = 2;
    for (int j0 = 1; j0 < w.part; j0 += kBatch) {
        float sv[kBatch][kN + 1];
#pragma unroll
        for (int q = 0; q < kBatch; ++q)
            if (j0 + q < w.part)
#pragma unroll
                for (int n = 0; n <= kN; ++n) sv[q][n] = __ldcg(rec + ((j0 + q) * (kN + 1) + n) * kLanes);
#pragma unroll
        for (int q = 0; q < kBatch; ++q)
            if (j0 + q < w.part)
#pragma unroll
                for (int n = 0; n < kN; ++n) h[n] = fmaf(fast_exp2(sv[q][kN] * a[n]), h[n], sv[q][n]);
    }
    return true;
}

// kMode 0: one item per CTA, one wave (plain and packed varlen launches, one
// CTA per unit: the straight-line form is 2 us faster on one-chunk items);
// 1: the split launch, (unit, part) items on a multi-wave grid, five CTAs per
// SM, a part waiting on the previous part's hand-off; 2: the fused
// chunk-parallel launch, whose one-wave cooperative grid walks items
// blockIdx.x, blockIdx.x + gridDim.x, ... (kLoop).  Thread 0 keeps kStages
// chunk loads in flight along the CTA's whole list, so the next item's first
// chunks arrive while the current item computes.
template <typename T, bool kBDL, bool kHasZ, bool kFullC, int kMode, int kR>
__global__ void __launch_bounds__(kLanes, bulk_min_blocks(kMode, kR, gate_mode(kHasZ, kR, kBDL, kMode) != 0)) bulk_kernel(const __grid_constant__ CUtensorMap tm_u,
                                                                  const __grid_constant__ CUtensorMap tm_d,
                                                                  const __grid_constant__ CUtensorMap tm_z,
                                                                  const __grid_constant__ CUtensorMap tm_b,
                                                                  const __grid_constant__ CUtensorMap tm_c,
                                                                  const __grid_constant__ CUtensorMap tm_y, BulkParams p) {
    pdl_wait();
    extern __shared__ unsigned char smem_raw[];
    constexpr int kZ = gate_mode(kHasZ, kR, kBDL, kMode);
    constexpr bool kZTile = kZ == 1;
    auto& sm = shared_window<Smem<T, kZ>>(smem_raw);
    const int tid = threadIdx.x;
    const unsigned long long D = p.channels;
    const int cw = kFullC ? kN : 1;
    const std::uint32_t c_bytes = static_cast<std::uint32_t>(cw) * kT * sizeof(T);
    constexpr bool kLoop = kMode != 0;
    const unsigned long long items = item_count(p);

    if (tid == 0) {
        prefetch_tensor_map(&tm_u);
        prefetch_tensor_map(&tm_d);
        prefetch_tensor_map(&tm_b);
        prefetch_tensor_map(&tm_c);
        prefetch_tensor_map(&tm_y);
        for (int s = 0; s < kStages; ++s) mbar_init(&sm.full[s], 1);
        if constexpr (kZ == 2) {
            prefetch_tensor_map(&tm_z);
            mbar_init(&sm.zfull[0], 1);
            mbar_init(&sm.zfull[1], 1);
        }
        fence_barrier_init();
        // First kStages loads of this CTA's (item, chunk) list.
        Cursor& c = sm.next;
        c.more = 1;
        c.it = blockIdx.x + p.item0;
        if (c.it >= items) {
            c.more = 0;
        } else {
            c.w = item_at<kBDL, kFullC>(p, c.it);
            c.chunk = c.w.c0 - 1;
            cursor_next<kBDL, kFullC>(c, p); // to the first chunk of the first item with chunks
        }
        for (int s = 0; s < kStages && c.more; ++s) {
            issue_chunk<T, kBDL, kHasZ, kR, kZ>(sm, s, static_cast<int>(c.w.tok0) + c.chunk * kT, c.w.row0, c.w.brow0, c.w.crow0,
                                            c.w.bb, c_bytes, &tm_u, &tm_d, &tm_z, &tm_b, &tm_c);
            cursor_next<kBDL, kFullC>(c, p);
        }
    }
    __syncthreads();

    bool fault = false;
    int gc = 0;    // chunks this CTA has consumed: stage gc % kStages, its (gc / kStages)-th use
    int gz = 0;    // kZ == 2: chunks whose gate halves this CTA has consumed (the halves' barrier parity)
    int pend = -1; // thread 0: the stage whose next load waits for its y store to read it
    const unsigned long long first = blockIdx.x + p.item0;
    const unsigned long long it_end = kLoop ? items : first + 1ull;
    for (unsigned long long it = first; it < it_end && (!kLoop || !fault); it += kLoop ? gridDim.x : 1u) {
        const Item w = item_at<kBDL, kFullC>(p, it);
        const unsigned long long d = w.d0 + tid, lane = w.b * D + d;
        // Per-lane constants: A * log2(e), D, dt bias; the state from h0 (or
        // zero) for a unit's first part, else from the previous part's hand-off.
        float a[kN], h[kN];
        load16(p.a + (p.a_shared ? 0 : d * kN), a, kLog2e);
        const float dskip = p.has_d ? p.d[d] : 0.0f;
        const float bias = p.bias ? p.bias[d] : 0.0f;
        const T* wrow = kR > 0 ? static_cast<const T*>(p.wdt) + d * (kR > 0 ? kR : 1) : nullptr;
        float dtsum = 0.0f; // sum of Delta over the part (chunk-parallel local pass)
        if (kMode == 2 && w.c1 == w.c0) continue; // a pass the fused mode skips
        if (w.part == 0) {
            if (p.h0) {
                load16(p.h0 + lane * kN, h);
            } else {
#pragma unroll
                for (int n = 0; n < kN; ++n) h[n] = 0.0f;
            }
        } else if (kMode == 2) {
            if (w.pass == 0) {
#pragma unroll
                for (int n = 0; n < kN; ++n) h[n] = 0.0f; // local pass from zero
            } else if (!fused_prefix(p, w, tid, a, h)) {
                fault = true;
                break;
            }
        } else if (p.phase == 1) {
#pragma unroll
            for (int n = 0; n < kN; ++n) h[n] = 0.0f; // local pass: from zero, corrected by the final pass
        } else if (p.phase == 2) {
            stash_load<T, kBDL>(p, w, d, h); // the part's true initial state, from the combine
        } else {
            bool ready = true;
            if (tid == 0) {
                const unsigned long long* f = flag_at<T, kBDL>(p, w, static_cast<unsigned long long>(w.c0) * kT);
                ready = false;
                for (std::uint32_t i = 0; i < (1u << 24); ++i) {
                    if (flag_acquire(f) == p.epoch) {
                        ready = true;
                        break;
                    }
                    __nanosleep(128);
                }
            }
            if (!__syncthreads_and(ready)) {
                fault = true;
                break;
            }
            stash_load<T, kBDL>(p, w, d, h);
        }

        // S4D-real A rows take the power-form decays; the choice is uniform
        // over the CTA, so the barriers inside the chunk loop stay uniform, and
        // every other A runs the exp-per-state loop unchanged.
        const bool pw = __syncthreads_and(s4d_row(p.a + (p.a_shared ? 0 : d * kN)));
        const float a0 = a[0];
        auto run_chunks = [&](auto pow_tag) {
            constexpr bool kPow = decltype(pow_tag)::value;
            for (int chunk = w.c0; chunk < w.c1; ++chunk, ++gc, ++gz) {
                const int s = gc % kStages;
                bool ok = mbar_wait_bounded(&sm.full[s], static_cast<std::uint32_t>((gc / kStages) & 1));
                if constexpr (kZ == 2) ok = mbar_wait_bounded(&sm.zfull[0], static_cast<std::uint32_t>(gz & 1)) && ok;
                if (!__syncthreads_and(ok)) {
                    fault = true;
                    break;
                }
                // B / C tiles to an FP32 token-major table.
                if (kBDL) {
                    // raw [state][token]: a thread takes 8 tokens of one state (16 bytes).
                    for (int i = tid; i < (kN + cw) * (kT / 8); i += kLanes) {
                        const int rowi = i / (kT / 8), t0 = (i % (kT / 8)) * 8;
                        const T* src = rowi < kN ? sm.braw[s] + rowi * kT + t0 : sm.craw[s] + (rowi - kN) * kT + t0;
                        const uint4 v = *reinterpret_cast<const uint4*>(src);
                        const std::uint32_t wv[4] = {v.x, v.y, v.z, v.w};
    #pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float2 f = unpack2<T>(wv[j]);
                            sm.bc[t0 + 2 * j][rowi] = f.x;
                            sm.bc[t0 + 2 * j + 1][rowi] = f.y;
                        }
                    }
                } else {
                    // raw [token][state]: already token-major.
                    for (int i = tid; i < kN * kT; i += kLanes) sm.bc[i / kN][i % kN] = to_f32(sm.braw[s][i]);
                    for (int i = tid; i < cw * kT; i += kLanes) sm.bc[i / cw][kN + i % cw] = to_f32(sm.craw[s][i]);
                }
                __syncthreads();

                // Tokens past the end of the sequence (zero-filled by the TMA, or the
                // next packed sequence) are not run through the recurrence.
                const unsigned long long left = w.len - static_cast<unsigned long long>(chunk) * kT;
                const int valid = static_cast<int>(left < kT ? left : kT);
                const int blocks8 = (valid + 7) / 8;
    #pragma unroll 1
                for (int q = 0; q < blocks8; ++q) {
                    if constexpr (kZ == 2) {
                        if (q == 2) {
                            // The gate's second half; past this barrier every thread is
                            // done with the first, which takes the next chunk's.
                            const bool zok = mbar_wait_bounded(&sm.zfull[1], static_cast<std::uint32_t>(gz & 1));
                            if (!__syncthreads_and(zok)) {
                                fault = true;
                                break;
                            }
                            if (tid == 0 && chunk + 1 < w.c1)
                                issue_gate_half<T, kBDL>(sm, 0, static_cast<int>(w.tok0) + (chunk + 1) * kT, w.row0, w.bb, &tm_z);
                        }
                    }
                    Block8 blk;
                    if constexpr (kBDL)
                        load_block_bdl<T, kHasZ, kZ == 2>(sm.u[s], sm.dl[s], kZ == 2 ? &sm.z[0][0] : sm.z[kHasZ ? s : 0], tid, q, blk);
                    else
                    {
                        load_block_bld<T, kHasZ, kZ != 0>(sm.u[s], sm.dl[s], kZ == 2 ? &sm.z[0][0] : sm.z[kZTile ? s : 0],
                                                          static_cast<const T*>(p.zg),
                                                         static_cast<unsigned long long>(w.bb) * p.length + w.tok0 +
                                                             static_cast<unsigned long long>(chunk) * kT,
                                                         p.zld, d, tid, q, valid - q * 8, blk);
                        if constexpr (kR > 0) delta_from_dt<T, kR>(sm.dl[s], wrow, q, blk);
                    }
                    float out[8];
                    if constexpr (kPow)
                        scan_block8_pow<kFullC, kHasZ, true, kMode != 1>(sm.bc, q, valid - q * 8, blk, a0, h, bias, dskip, p.softplus,
                                                                        out, dtsum);
                    else
                        scan_block8<kFullC, kHasZ, true, kMode != 1>(sm.bc, q, valid - q * 8, blk, a, h, bias, dskip, p.softplus, out,
                                                                    dtsum);
                    if (kBDL) store_block_bdl<T>(sm.u[s], tid, q, out);
                    else store_block_bld<T>(sm.u[s], tid, q, out);
                    if (q == 0 && tid == 0 && pend >= 0) {
                        // The previous chunk's stage, once its y store has read it:
                        // the chunk kStages after that one.  A token block into this
                        // chunk, the store has had time to drain.
                        bulk_wait_read<0>();
                        Cursor& c = sm.next;
                        issue_chunk<T, kBDL, kHasZ, kR, kZ>(sm, pend, static_cast<int>(c.w.tok0) + c.chunk * kT, c.w.row0, c.w.brow0,
                                                        c.w.crow0, c.w.bb, c_bytes, &tm_u, &tm_d, &tm_z, &tm_b, &tm_c);
                        cursor_next<kBDL, kFullC>(c, p);
                        pend = -1;
                    }
                }
                if (fault) break;
                if constexpr (kZ == 2) {
                    if (blocks8 <= 2) {
                        // A short last chunk: its gate's second half arrived unread.
                        const bool zok = mbar_wait_bounded(&sm.zfull[1], static_cast<std::uint32_t>(gz & 1));
                        if (!__syncthreads_and(zok)) {
                            fault = true;
                            break;
                        }
                    }
                }
                fence_async_shared();
                __syncthreads();
                const int tc0 = static_cast<int>(w.tok0) + chunk * kT;
                // Local-pass outputs (parts after the first) are not final.
                const bool write_y = !((p.phase == 1 || (kMode == 2 && w.pass == 0)) && w.part > 0);
                const bool tail = !kBDL && p.cu && valid < kT;
                if (tail && write_y) {
                    // A packed sequence's partial last chunk: a tile store would also
                    // write the next sequence's rows, so store the valid rows only.
                    T* yg = static_cast<T*>(p.y);
                    for (int t = 0; t < valid; ++t) yg[(static_cast<unsigned long long>(tc0) + t) * D + d] = sm.u[s][t * kLanes + tid];
                }
                if (tid == 0) {
                    if (!tail && write_y) {
                        if (kBDL) tma_store_2d(&tm_y, sm.u[s], tc0, w.row0);
                        else tma_store_3d(&tm_y, sm.u[s], w.row0, tc0, w.bb);
                    }
                    bulk_commit();
                    if constexpr (kZ == 2) {
                        // The next chunk's gate: the second half (all of it after a
                        // short chunk, whose first half was not taken mid-chunk).
                        if (chunk + 1 < w.c1) {
                            if (blocks8 <= 2) issue_gate_half<T, kBDL>(sm, 0, tc0 + kT, w.row0, w.bb, &tm_z);
                            issue_gate_half<T, kBDL>(sm, 1, tc0 + kT, w.row0, w.bb, &tm_z);
                        }
                    }
                    // Stage s takes the chunk kStages ahead in this CTA's list once
                    // the store above has read it (first token block of the next chunk).
                    if (sm.next.more) pend = s;
                }
            }
        };
        if constexpr (kZ == 2) {
            // The gate of the item's first chunk (later chunks' halves load while
            // the chunk before them computes).
            if (tid == 0 && w.c1 > w.c0) {
                const int t0z = static_cast<int>(w.tok0) + w.c0 * kT;
                issue_gate_half<T, kBDL>(sm, 0, t0z, w.row0, w.bb, &tm_z);
                issue_gate_half<T, kBDL>(sm, 1, t0z, w.row0, w.bb, &tm_z);
            }
        }
        if (pw) run_chunks(std::true_type{});
        else run_chunks(std::false_type{});
        if (fault) break;
        if (kMode == 2) {
            if (w.pass == 0) {
                // Local pass: the part's end state and its sum of Delta to the
                // scratch, then this part's flag.
                float* out = p.scratch + (static_cast<unsigned long long>(w.b * (D / kLanes) + w.d0 / kLanes) * p.parts + w.part) *
                                             (kN + 1) * kLanes + tid;
#pragma unroll
                for (int n = 0; n < kN; ++n) out[n * kLanes] = h[n];
                out[kN * kLanes] = dtsum;
                __threadfence();
                __syncthreads();
                if (tid == 0) flag_release(fused_flag(p, w, w.part), p.epoch);
            } else if (p.h_final && w.part + 1 == p.parts) {
                store16(p.h_final + lane * kN, h);
            }
        } else if (p.phase == 1) {
            // Local pass: the part's end state and its sum of Delta go to the
            // next part's first outputs for the combine (the last part's are
            // not needed).
            if (w.part + 1 < p.parts) stash_store<T, kBDL>(p, w, d, h, dtsum);
        } else if (p.phase == 0 && !w.last) {
            // Hand the state to the unit's next part.
            stash_store<T, kBDL>(p, w, d, h);
            __threadfence();
            __syncthreads();
            if (tid == 0) flag_release(flag_at<T, kBDL>(p, w, static_cast<unsigned long long>(w.c1) * kT), p.epoch);
        } else if (p.h_final && w.last) {
            store16(p.h_final + lane * kN, h);
        }
    }
    if (fault) {
        if (tid == 0) {
            atomicOr(&g_bulk_fault, 1u);
            // Give copies still in flight a bounded chance to land before the
            // CTA's shared memory is released.
            for (int s = 0; s < kStages; ++s) (void)mbar_wait_bounded(&sm.full[s], 0u, 1u << 16);
            if constexpr (kZ == 2)
                for (int h2 = 0; h2 < 2; ++h2) (void)mbar_wait_bounded(&sm.zfull[h2], 0u, 1u << 16);
        }
        return;
    }
    if (tid == 0) bulk_wait<0>();
}

// ------------------------------------------------------------ quad variant
// Four threads per lane, four of the 16 states each, for launches that leave
// the SMs mostly empty (few units; the fused chunk-parallel launch): 16 warps
// per CTA instead of 4, so a lane's per-token dependency chain is spread over
// four threads.  Thread q of a lane forms Delta for tokens q and q + 4 of every
// eight and the four threads exchange them by shuffles; the partial sums
// C_n h_n of the four state quarters meet by two xor shuffles; thread q
// stores tokens q and q + 4.  (B, L, D) layout with a full-width C, dense rows
// or packed varlen sequences; modes 0 (one item per CTA) and 2 (fused
// chunk-parallel, with scratch).
constexpr int kQ = 4;         // threads per lane
constexpr int kQS = kN / kQ;  // states per thread
static_assert(kQS == 4, "the quad kernel moves a thread's states as one float4");

// quad form of fused_prefix: this thread's kQS states of the lane.
__device__ __forceinline__ bool quad_prefix(const BulkParams& p, const Item& w, int tid, int li, int n0, const float (&a)[kQS],
                                            float (&h)[kQS]) {
    bool ready = true;
    if (tid < w.part) {
        const unsigned long long* f = fused_flag(p, w, tid);
        ready = false;
        for (std::uint32_t i = 0; i < (1u << 24); ++i) {
            if (flag_acquire(f) == p.epoch) {
                ready = true;
                break;
            }
            __nanosleep(64);
        }
    }
    if (!__syncthreads_and(ready)) return false;
    const unsigned long long unit = w.b * (p.channels / kLanes) + w.d0 / kLanes;
    const float* rec = p.scratch + unit * p.parts * (kN + 1) * kLanes + li;
#pragma unroll
    for (int n = 0; n < kQS; ++n) h[n] = __ldcg(rec + (n0 + n) * kLanes); // S_0
    constexpr int kBatch = 2;
    for (int j0 = 1; j0 < w.part; j0 += kBatch) {
        float sv[kBatch][kQS + 1];
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
            if (j0 + b < w.part) {
                const float* r = rec + static_cast<unsigned long long>(j0 + b) * (kN + 1) * kLanes;
#pragma unroll
                for (int n = 0; n < kQS; ++n) sv[b][n] = __ldcg(r + (n0 + n) * kLanes);
                sv[b][kQS] = __ldcg(r + kN * kLanes);
            }
        }
#pragma unroll
        for (int b = 0; b < kBatch; ++b)
            if (j0 + b < w.part)
#pragma unroll
                for (int n = 0; n < kQS; ++n) h[n] = fmaf(fast_exp2(sv[b][kQS] * a[n]), h[n], sv[b][n]);
    }
    return true;
}

template <typename T, bool kHasZ, int kMode, int kR>
__global__ void __launch_bounds__(kLanes * kQ, 2) quad_kernel(const __grid_constant__ CUtensorMap tm_u,
                                                             const __grid_constant__ CUtensorMap tm_d,
                                                             const __grid_constant__ CUtensorMap tm_z,
                                                             const __grid_constant__ CUtensorMap tm_b,
                                                             const __grid_constant__ CUtensorMap tm_c,
                                                             const __grid_constant__ CUtensorMap tm_y, BulkParams p) {
    pdl_wait();
    extern __shared__ unsigned char smem_raw[];
    auto& sm = shared_window<SmemY<T>>(smem_raw);
    const int tid = threadIdx.x, li = tid / kQ, q = tid % kQ, n0 = q * kQS;
    const int quad0 = (tid & 31) & ~(kQ - 1); // this quad's first lane in the warp
    const unsigned long long D = p.channels;
    const std::uint32_t c_bytes = kN * kT * sizeof(T);
    constexpr bool kLoop = kMode != 0;
    const unsigned long long items = p.units * static_cast<unsigned long long>(p.parts) * (kMode == 2 ? 2u : 1u);

    if (tid == 0) {
        prefetch_tensor_map(&tm_u);
        prefetch_tensor_map(&tm_d);
        prefetch_tensor_map(&tm_b);
        prefetch_tensor_map(&tm_c);
        prefetch_tensor_map(&tm_y);
        for (int s = 0; s < kStages; ++s) mbar_init(&sm.full[s], 1);
        fence_barrier_init();
        Cursor& c = sm.next;
        c.more = 1;
        c.it = blockIdx.x + p.item0;
        if (c.it >= items) {
            c.more = 0;
        } else {
            c.w = item_at<false, true>(p, c.it);
            c.chunk = c.w.c0 - 1;
            cursor_next<false, true>(c, p);
        }
        for (int s = 0; s < kStages && c.more; ++s) {
            issue_chunk<T, false, kHasZ, kR>(sm, s, static_cast<int>(c.w.tok0) + c.chunk * kT, c.w.row0, c.w.brow0, c.w.crow0,
                                             c.w.bb, c_bytes, &tm_u, &tm_d, &tm_z, &tm_b, &tm_c);
            cursor_next<false, true>(c, p);
        }
    }
    __syncthreads();

    bool fault = false;
    int gc = 0;
    const unsigned long long first = blockIdx.x + p.item0;
    const unsigned long long it_end = kLoop ? items : first + 1ull;
    for (unsigned long long it = first; it < it_end && (!kLoop || !fault); it += kLoop ? gridDim.x : 1u) {
        const Item w = item_at<false, true>(p, it);
        if (kMode == 2 && w.c1 == w.c0) continue; // a pass the fused mode skips
        const unsigned long long d = w.d0 + li, lane = w.b * D + d;
        float a[kQS], h[kQS];
        {
            const float4 av = __ldg(reinterpret_cast<const float4*>(p.a + (p.a_shared ? 0 : d * kN) + n0));
            a[0] = av.x * kLog2e; a[1] = av.y * kLog2e; a[2] = av.z * kLog2e; a[3] = av.w * kLog2e;
        }
        const float dskip = p.has_d ? p.d[d] : 0.0f;
        const float bias = p.bias ? p.bias[d] : 0.0f;
        const T* wrow = kR > 0 ? static_cast<const T*>(p.wdt) + d * (kR > 0 ? kR : 1) : nullptr;
        float dtsum = 0.0f;
        if (w.part == 0) {
            const float4 hv = p.h0 ? __ldg(reinterpret_cast<const float4*>(p.h0 + lane * kN + n0)) : make_float4(0.f, 0.f, 0.f, 0.f);
            h[0] = hv.x; h[1] = hv.y; h[2] = hv.z; h[3] = hv.w;
        } else if (w.pass == 0) {
#pragma unroll
            for (int n = 0; n < kQS; ++n) h[n] = 0.0f; // fused local pass from zero
        } else if (!quad_prefix(p, w, tid, li, n0, a, h)) {
            fault = true;
            break;
        }

        for (int chunk = w.c0; chunk < w.c1; ++chunk, ++gc) {
            const int s = gc % kStages;
            const bool ok = mbar_wait_bounded(&sm.full[s], static_cast<std::uint32_t>((gc / kStages) & 1));
            if (tid == 0) bulk_wait_read<0>();
            if (!__syncthreads_and(ok)) {
                fault = true;
                break;
            }
            for (int i = tid; i < kN * kT; i += kLanes * kQ) sm.bc[i / kN][i % kN] = to_f32(sm.braw[s][i]);
            for (int i = tid; i < kN * kT; i += kLanes * kQ) sm.bc[i / kN][kN + i % kN] = to_f32(sm.craw[s][i]);
            __syncthreads();

            const unsigned long long left = w.len - static_cast<unsigned long long>(chunk) * kT;
            const int valid = static_cast<int>(left < kT ? left : kT);
            const int blocks8 = (valid + 7) / 8;
            const unsigned long long zrow0 = static_cast<unsigned long long>(w.bb) * p.length + w.tok0 +
                                             static_cast<unsigned long long>(chunk) * kT;
#pragma unroll 1
            for (int qb = 0; qb < blocks8; ++qb) {
                const int count = valid - qb * 8;
                float u8[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) u8[j] = to_f32(sm.u[s][(qb * 8 + j) * kLanes + li]);
                // Delta of tokens q and q + 4.
                float dtq[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int t = qb * 8 + q + 4 * e;
                    float x;
                    if constexpr (kR > 0) {
                        const uint4* row = reinterpret_cast<const uint4*>(sm.dl[s] + t * kR);
                        const uint4* wr = reinterpret_cast<const uint4*>(wrow);
                        float acc = 0.0f;
#pragma unroll
                        for (int v = 0; v < kR / 8; ++v) {
                            const uint4 d8 = row[v], w8 = __ldg(wr + v);
                            const std::uint32_t dd[4] = {d8.x, d8.y, d8.z, d8.w}, ww[4] = {w8.x, w8.y, w8.z, w8.w};
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const float2 fd = unpack2<T>(dd[i]), fw = unpack2<T>(ww[i]);
                                acc = fmaf(fd.x, fw.x, acc);
                                acc = fmaf(fd.y, fw.y, acc);
                            }
                        }
                        x = acc;
                    } else {
                        x = to_f32(sm.dl[s][t * kLanes + li]);
                    }
                    const float v = x + bias;
                    dtq[e] = p.softplus ? softplus_poly(v) : v;
                }
                float yp[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float dt = __shfl_sync(0xffffffffu, dtq[j / 4], quad0 + (j % 4));
                    yp[j] = 0.0f;
                    if (j < count) { // tokens past the end stay out of the state
                        dtsum += dt;
                        const float du = dt * u8[j];
                        const float4 bq = *reinterpret_cast<const float4*>(&sm.bc[qb * 8 + j][n0]);
                        const float4 cq = *reinterpret_cast<const float4*>(&sm.bc[qb * 8 + j][kN + n0]);
                        const float bb[4] = {bq.x, bq.y, bq.z, bq.w}, cc[4] = {cq.x, cq.y, cq.z, cq.w};
                        float acc[4];
#pragma unroll
                        for (int n = 0; n < kQS; ++n) {
                            h[n] = fmaf(fast_exp2(dt * a[n]), h[n], du * bb[n]);
                            acc[n] = cc[n] * h[n];
                        }
                        yp[j] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
                    }
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    yp[j] += __shfl_xor_sync(0xffffffffu, yp[j], 1);
                    yp[j] += __shfl_xor_sync(0xffffffffu, yp[j], 2);
                }
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int j = q + 4 * e, t = qb * 8 + j;
                    float y = 0.0f;
                    if (j < count) {
                        y = fmaf(dskip, u8[j], yp[j]);
                        if constexpr (kHasZ)
                            y *= silu(to_f32(static_cast<const T*>(p.zg)[(zrow0 + static_cast<unsigned long long>(t)) * p.zld + d]));
                    }
                    sm.y[t * kLanes + li] = from_f32<T>(y);
                }
            }
            fence_async_shared();
            __syncthreads();
            const int tc0 = static_cast<int>(w.tok0) + chunk * kT;
            const bool write_y = !(kMode == 2 && w.pass == 0 && w.part > 0); // local-pass outputs are not final
            const bool tail = p.cu && valid < kT;
            if (tail && write_y) {
                T* yg = static_cast<T*>(p.y);
                for (int t = q; t < valid; t += kQ) yg[(static_cast<unsigned long long>(tc0) + t) * D + d] = sm.y[t * kLanes + li];
            }
            if (tid == 0) {
                if (!tail && write_y) tma_store_3d(&tm_y, sm.y, w.row0, tc0, w.bb);
                bulk_commit();
                Cursor& c = sm.next;
                if (c.more) {
                    issue_chunk<T, false, kHasZ, kR>(sm, s, static_cast<int>(c.w.tok0) + c.chunk * kT, c.w.row0, c.w.brow0,
                                                     c.w.crow0, c.w.bb, c_bytes, &tm_u, &tm_d, &tm_z, &tm_b, &tm_c);
                    cursor_next<false, true>(c, p);
                }
            }
        }
        if (fault) break;
        if (kMode == 2 && w.pass == 0) {
            float* rec = p.scratch + (static_cast<unsigned long long>(w.b * (D / kLanes) + w.d0 / kLanes) * p.parts + w.part) *
                                         (kN + 1) * kLanes + li;
#pragma unroll
            for (int n = 0; n < kQS; ++n) rec[(n0 + n) * kLanes] = h[n];
            if (q == 0) rec[kN * kLanes] = dtsum;
            __threadfence();
            __syncthreads();
            if (tid == 0) flag_release(fused_flag(p, w, w.part), p.epoch);
        } else if (p.h_final && w.part + 1 == p.parts) {
            *reinterpret_cast<float4*>(p.h_final + lane * kN + n0) = make_float4(h[0], h[1], h[2], h[3]);
        }
    }
    if (fault) {
        if (tid == 0) {
            atomicOr(&g_bulk_fault, 1u);
            for (int s = 0; s < kStages; ++s) (void)mbar_wait_bounded(&sm.full[s], 0u, 1u << 16);
        }
        return;
    }
    if (tid == 0) bulk_wait<0>();
}

// ------------------------------------------------------------ wait probe
// Diagnostics for the bounded waits: one CTA waits on a hand-off flag that
// nothing sets and on an mbarrier nothing arrives at, with the scan kernels'
// own wait helpers, `limit` polls each; on time-out it sets the fault word,
// as the scan kernels do, and returns (the context stays usable).
__device__ unsigned long long g_probe_flag; // never written

__global__ void wait_probe_kernel(std::uint32_t limit) {
    __shared__ alignas(8) std::uint64_t bar;
    if (threadIdx.x != 0) return;
    bool ok = false;
    for (std::uint32_t i = 0; i < limit; ++i) {
        if (flag_acquire(&g_probe_flag) == 1ull) {
            ok = true;
            break;
        }
        __nanosleep(128);
    }
    mbar_init(&bar, 1);
    fence_barrier_init();
    const bool arrived = mbar_wait_bounded(&bar, 0u, limit);
    if (!ok || !arrived) atomicOr(&g_bulk_fault, 1u);
}

// ---------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// 3D map (inner, mid, outer) with a (box_inner, box_mid, 1) box, no swizzle;
// consecutive mid rows `row_stride` elements apart (0: dense, = inner).
bool make_map_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, unsigned long long inner,
                 unsigned long long mid, unsigned long long outer, unsigned box_inner, unsigned box_mid,
                 unsigned long long row_stride = 0) {
    auto fn = encode_fn();
    if (!fn) return false;
    const unsigned long long rs = row_stride ? row_stride : inner;
    const cuuint64_t dims[3] = {inner, mid, outer};
    const cuuint64_t strides[2] = {rs * 2, rs * mid * 2};
    const cuuint32_t box[3] = {box_inner, box_mid, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, unsigned long long inner,
                 unsigned long long rows, unsigned long long row_stride_bytes, unsigned box_inner, unsigned box_rows,
                 CUtensorMapSwizzle swizzle) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T, bool kBDL, bool kHasZ, bool kFullC, int kMode, int kR = 0>
struct Variant {
    static const void* fn() { return reinterpret_cast<const void*>(bulk_kernel<T, kBDL, kHasZ, kFullC, kMode, kR>); }
    static cudaError_t prepare() {
        static std::atomic<int> done[64];
        return once_per_device(done, [] {
            return cudaFuncSetAttribute(fn(), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem_bytes<Smem<T, gate_mode(kHasZ, kR, kBDL, kMode)>>()));
        });
    }
    static size_t smem() { return smem_bytes<Smem<T, gate_mode(kHasZ, kR, kBDL, kMode)>>(); }
};

// Chunk-parallel combine, one thread per (batch row, channel): the local
// pass left each part k < K - 1's end state S_k (from zero; part 0 from h0)
// and its sum of Delta at part k + 1's first outputs.  Over the parts in
// order the true initial state of part k is H_1 = S_0 and
// H_k = exp(A * sum Delta_{k-1}) H_{k-1} + S_{k-1} (the recurrence is linear in
// h and the decays of a part multiply to one exponential), written back in
// place for the final pass.
template <typename T, bool kBDL>
__global__ void __launch_bounds__(256) combine_kernel(BulkParams p, unsigned long long rows) {
    pdl_wait();
    const unsigned long long idx = static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= rows * p.channels) return;
    const unsigned long long d = idx % p.channels;
    Item w{};
    w.b = idx / p.channels;
    float a[kN], h[kN], s[kN];
    const float* arow = p.a + (p.a_shared ? 0 : d * kN);
#pragma unroll
    for (int n = 0; n < kN; ++n) a[n] = arow[n] * kLog2e;
    for (int k = 1; k < p.parts; ++k) {
        w.c0 = k * p.nchunks / p.parts;
        if (k == 1) {
            stash_load<T, kBDL>(p, w, d, h); // part 0 ran from h0: already the true state
            continue;
        }
        stash_load<T, kBDL>(p, w, d, s);
        const float sum = stash_extra<T, kBDL>(p, w, d);
#pragma unroll
        for (int n = 0; n < kN; ++n) h[n] = fmaf(fast_exp2(sum * a[n]), h[n], s[n]);
        stash_put<T, kBDL>(p, stash_at<T, kBDL>(p, w, d, static_cast<unsigned long long>(w.c0) * kT), h, nullptr);
    }
}

struct Pick {
    const void* fn;
    size_t smem;
    cudaError_t (*prepare)();
    int threads = kLanes; // threads per CTA the variant launches with
};

template <typename T, bool kBDL, bool kHasZ, bool kFullC>
Pick make_pick(int mode) {
    if (mode == 1) {
        using V = Variant<T, kBDL, kHasZ, kFullC, 1>;
        return {V::fn(), V::smem(), &V::prepare};
    }
    if (mode == 2) {
        using V = Variant<T, kBDL, kHasZ, kFullC, 2>;
        return {V::fn(), V::smem(), &V::prepare};
    }
    using V = Variant<T, kBDL, kHasZ, kFullC, 0>;
    return {V::fn(), V::smem(), &V::prepare};
}

template <typename T, bool kBDL>
Pick pick_z(bool z, bool full_c, int mode) {
    if (z) return full_c ? make_pick<T, kBDL, true, true>(mode) : make_pick<T, kBDL, true, false>(mode);
    return full_c ? make_pick<T, kBDL, false, true>(mode) : make_pick<T, kBDL, false, false>(mode);
}

// mode 0: one item per CTA; 1: split launch; 2: fused chunk-parallel launch.
Pick pick(int dtype, bool bdl, bool z, bool full_c, int mode) {
    if (dtype == SACC_DTYPE_BF16)
        return bdl ? pick_z<__nv_bfloat16, true>(z, full_c, mode) : pick_z<__nv_bfloat16, false>(z, full_c, mode);
    return bdl ? pick_z<__half, true>(z, full_c, mode) : pick_z<__half, false>(z, full_c, mode);
}

// The variants that form delta in the scan from dt rows of rank kR (the
// block's (B, L, D) layout with a gate and a full-width C).
template <typename T, int kR>
Pick make_pick_dt(int mode) {
    if (mode == 1) {
        using V = Variant<T, false, true, true, 1, kR>;
        return {V::fn(), V::smem(), &V::prepare};
    }
    if (mode == 2) {
        using V = Variant<T, false, true, true, 2, kR>;
        return {V::fn(), V::smem(), &V::prepare};
    }
    using V = Variant<T, false, true, true, 0, kR>;
    return {V::fn(), V::smem(), &V::prepare};
}

Pick pick_dt(int dtype, int rank, int mode) {
    if (dtype == SACC_DTYPE_BF16) return rank == 8 ? make_pick_dt<__nv_bfloat16, 8>(mode) : make_pick_dt<__nv_bfloat16, 16>(mode);
    return rank == 8 ? make_pick_dt<__half, 8>(mode) : make_pick_dt<__half, 16>(mode);
}

template <typename T, bool kHasZ, int kMode, int kR>
struct QuadVariant {
    static const void* fn() { return reinterpret_cast<const void*>(quad_kernel<T, kHasZ, kMode, kR>); }
    static cudaError_t prepare() {
        static std::atomic<int> done[64];
        return once_per_device(done, [] {
            return cudaFuncSetAttribute(fn(), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem_bytes<SmemY<T>>()));
        });
    }
    static size_t smem() { return smem_bytes<SmemY<T>>(); }
};

template <typename T, bool kHasZ, int kR>
Pick make_pick_quad(int mode) {
    if (mode == 2) {
        using V = QuadVariant<T, kHasZ, 2, kR>;
        return {V::fn(), V::smem(), &V::prepare, kLanes * kQ};
    }
    using V = QuadVariant<T, kHasZ, 0, kR>;
    return {V::fn(), V::smem(), &V::prepare, kLanes * kQ};
}

template <typename T>
Pick pick_quad_t(bool z, int rank, int mode) {
    if (rank == 8) return make_pick_quad<T, true, 8>(mode);
    if (rank == 16) return make_pick_quad<T, true, 16>(mode);
    return z ? make_pick_quad<T, true, 0>(mode) : make_pick_quad<T, false, 0>(mode);
}

// The four-threads-per-lane variant ((B, L, D), full-width C; modes 0 and 2).
Pick pick_quad(const SaccScanExArgs& a, const DtFusion* dtf, int mode) {
    const int rank = dtf ? dtf->rank : 0;
    return a.dtype == SACC_DTYPE_BF16 ? pick_quad_t<__nv_bfloat16>(a.z != nullptr, rank, mode)
                                      : pick_quad_t<__half>(a.z != nullptr, rank, mode);
}

bool quad_eligible(const SaccScanExArgs& a) { return a.layout == SACC_LAYOUT_BLD && a.c_width == kN; }

// The variant for this call and mode.
Pick pick_for(const SaccScanExArgs& a, const DtFusion* dtf, int mode) {
    if (dtf) return pick_dt(a.dtype, dtf->rank, mode);
    return pick(a.dtype, a.layout == SACC_LAYOUT_BDL, a.z != nullptr, a.c_width != 1, mode);
}

bool aligned16(const void* p) { return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0; }

// CTAs of a variant resident at once on the current device (SMs x CTAs per
// SM at the variant's own block size), queried once per (variant, device).
unsigned long long resident_ctas(const Pick& k) {
    struct Entry {
        const void* fn;
        int dev;
        unsigned long long ctas;
    };
    static std::mutex mu;
    static Entry cache[64];
    static int used = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        for (int i = 0; i < used; ++i)
            if (cache[i].fn == k.fn && cache[i].dev == dev) return cache[i].ctas;
    }
    int sms = 148, per_sm = 1;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k.fn, k.threads, k.smem) != cudaSuccess || per_sm < 1) per_sm = 1;
    const unsigned long long ctas = static_cast<unsigned long long>(sms) * static_cast<unsigned long long>(per_sm);
    std::lock_guard<std::mutex> lock(mu);
    if (used < 64) cache[used++] = Entry{k.fn, dev, ctas};
    return ctas;
}

// Parts per unit for a launch of more units than one wave of the one-item
// kernel holds: enough (unit, part) items for about four waves of `wave`
// resident CTAs, P = ceil(4 wave / units), at most 8 and at most half the
// chunks (each part keeps two chunks; with L % 8 == 0 the last one keeps at
// least 40 tokens, the hand-off's 36).  The items are part-major, one per
// CTA, so CTAs that finish early take new parts while the rest of their SM is
// still busy: the warp scheduler favours an SM's oldest CTAs (measured on
// B200: the first of five runs 2.8 times faster than the last), and a one-wave
// walk would leave each SM with ever fewer CTAs at its end.  Measured at
// (B, D, L) = (64, 1536, 2048): P = 4 gives 1576 GB/s against 1482 for equal
// one-wave ranges and 1285 unsplit.
int split_parts(unsigned long long units, unsigned long long wave, int nchunks, unsigned long long length) {
    if (wave == 0 || length % 8 != 0) return 1;
    unsigned long long P = (4 * wave + units - 1) / units;
    if (P > 8) P = 8;
    if (P > static_cast<unsigned long long>(nchunks / 2)) P = static_cast<unsigned long long>(nchunks / 2);
    return P < 1 ? 1 : static_cast<int>(P);
}

// Parts for the chunk-parallel mode (a local pass over all parts, a combine,
// a final pass over parts 1..K-1): for launches that leave most SMs idle
// (units at most a quarter of the SMs), sequences of at least four chunks and
// L % 8 == 0 (each part keeps >= 2 chunks, the stash 34 tokens).  K fills the
// SMs with one part per SM in the local pass; 0 when the mode does not apply.
int chunk_parts(unsigned long long units, unsigned long long sms, int nchunks, unsigned long long length) {
    if (units == 0 || units * 4 > sms || nchunks < 4 || length % 8 != 0) return 0;
    unsigned long long k = sms / units;
    if (k > static_cast<unsigned long long>(nchunks / 2)) k = static_cast<unsigned long long>(nchunks / 2);
    if (k > 32) k = 32;
    return k >= 3 ? static_cast<int>(k) : 0; // two passes over 2/K of the sequence: below 3 parts no gain
}

// Parts for the fused chunk-parallel mode (one cooperative launch with a
// scratch buffer for the parts' records, so parts of one chunk are allowed
// and any L): launches that leave most SMs idle (units at most a quarter of
// the SMs), K = as many whole-chunk parts as resident CTAs allow (at most 32),
// when two passes over the longest part plus about one chunk of hand-off
// beat the sequential walk; 0 when the mode does not apply.
int fused_parts(unsigned long long units, unsigned long long sms, unsigned long long wave, int nchunks) {
    if (units == 0 || units * 4 > sms || nchunks < 4) return 0;
    unsigned long long k = wave / units;
    if (k > static_cast<unsigned long long>(nchunks)) k = static_cast<unsigned long long>(nchunks);
    if (k > static_cast<unsigned long long>(kMaxFusedParts)) k = kMaxFusedParts;
    if (k < 2) return 0;
    const unsigned long long longest = (static_cast<unsigned long long>(nchunks) + k - 1) / k;
    return 2 * longest + 1 < static_cast<unsigned long long>(nchunks) ? static_cast<int>(k) : 0;
}

std::size_t fused_scratch_bytes(unsigned long long units, int parts) {
    return static_cast<std::size_t>(units) * static_cast<std::size_t>(parts) * ((kN + 1) * kLanes * sizeof(float) + 8);
}

// A value no earlier split launch of this process used, never zero: the
// hand-off flags in the output are compared against it.
unsigned long long next_epoch() {
    static std::atomic<unsigned long long> counter{0};
    static const unsigned long long salt = [] {
        std::random_device rd;
        return (static_cast<unsigned long long>(rd()) << 32) ^ rd() ^ 0x9E3779B97F4A7C15ull;
    }();
    unsigned long long v = 0;
    while (v == 0) v = (counter.fetch_add(1) + 1) * 0xD6E8FEB86659FD93ull ^ salt;
    return v;
}

} // namespace

// The bulk kernel's domain: 16-bit activations, N = 16, channels in 128-wide
// tiles inside one group, 16-byte aligned tensors and 16-byte row strides for
// the TMA ((B, D, L): L % 8 == 0; (B, L, D): a full-width C, whose rows are
// then 16 * groups * 2 bytes, any L, packed varlen sequences too).  Other
// calls use the general kernel.
bool bulk_eligible(const SaccScanExArgs& a, const RowStrides* rs) {
    if (rs) {
        // Strided z / B / C rows (the block's fused projection outputs): dense
        // (B, L, D) rows only, 16-byte row pitches, rows at least as wide as the data.
        const unsigned long long cw = a.c_width;
        if (a.layout != SACC_LAYOUT_BLD || a.cu_seqlens != nullptr || (rs->z && (rs->z < a.channels || rs->z % 8)) ||
            (rs->b && (rs->b < a.groups * kN || rs->b % 8)) || (rs->c && (rs->c < a.groups * cw || rs->c % 8)))
            return false;
    }
    if ((a.dtype != SACC_DTYPE_BF16 && a.dtype != SACC_DTYPE_F16) || a.state != kN || a.length == 0 || a.groups == 0 ||
        a.channels % kLanes != 0 || (a.channels / a.groups) % kLanes != 0)
        return false;
    if (a.cu_seqlens != nullptr) {
        // Packed varlen: (B, L, D) with batch 1, any sequence lengths.
        if (a.layout != SACC_LAYOUT_BLD || a.batch != 1 || a.c_width != kN || a.channels % 8 != 0 || a.nseq <= 0 ||
            static_cast<unsigned long long>(a.nseq) * (a.channels / kLanes) > 0x7fffffffull)
            return false;
    } else if (a.layout == SACC_LAYOUT_BDL) {
        if (a.length % 8 != 0) return false;
    } else if (a.layout == SACC_LAYOUT_BLD) {
        // Any length: the 3D maps stop at L (tokens past it read zero and are
        // kept out of the state; the y store stops at L).
        if (a.c_width != kN || a.channels % 8 != 0) return false;
    } else {
        return false;
    }
    for (const void* ptr : {a.u, a.delta, a.b, a.c, a.z, static_cast<const void*>(a.y), static_cast<const void*>(a.a),
                            static_cast<const void*>(a.h0), static_cast<const void*>(a.h_final)})
        if (ptr && !aligned16(ptr)) return false;
    const unsigned long long rows = a.batch * a.channels, tokens = a.batch * a.length;
    return rows <= 0x7fffffffull && tokens <= 0x7fffffffull && a.batch * a.groups * kN <= 0x7fffffffull;
}

namespace {
// Parts of the fused chunk-parallel mode for this call on the current device
// (0: it does not apply), and the variant it would use.
int fused_plan(const SaccScanExArgs& a, const DtFusion* dtf, Pick& k) {
    if (a.cu_seqlens != nullptr) return 0;
    k = quad_eligible(a) ? pick_quad(a, dtf, 2) : pick_for(a, dtf, 2);
    if (k.prepare() != cudaSuccess) return 0;
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const unsigned long long units = a.batch * (a.channels / kLanes);
    return fused_parts(units, static_cast<unsigned long long>(sms), resident_ctas(k),
                       static_cast<int>((a.length + kT - 1) / kT));
}
} // namespace

bool dt_fusable(const SaccScanExArgs& a, const DtFusion& f) {
    return (f.rank == 8 || f.rank == 16) && a.layout == SACC_LAYOUT_BLD && a.cu_seqlens == nullptr && a.z != nullptr &&
           a.c_width == kN && f.dt != nullptr && f.w != nullptr && aligned16(f.dt) && aligned16(f.w) &&
           f.ld >= static_cast<unsigned long long>(f.rank) && f.ld % 8 == 0;
}

ZeroSpan bulk_scan_flags(void* scratch, std::size_t scratch_bytes) {
    // units x parts x (17 x 128 FP32 record + 8-byte flag), flags last.
    const std::size_t per = (kN + 1) * kLanes * sizeof(float) + 8, items = scratch_bytes / per;
    ZeroSpan z;
    if (scratch != nullptr && items > 0) {
        z.ptr = reinterpret_cast<unsigned long long*>(static_cast<unsigned char*>(scratch) + items * (per - 8));
        z.words = items;
    }
    return z;
}

std::size_t bulk_scan_scratch_bytes(const SaccScanExArgs& a, const DtFusion* dtf) {
    Pick k{};
    const int parts = fused_plan(a, dtf, k);
    return parts ? fused_scratch_bytes(a.batch * (a.channels / kLanes), parts) : 0;
}

cudaError_t launch_scan_bulk(const SaccScanExArgs& a, cudaStream_t stream, const RowStrides* rs, void* scratch,
                             std::size_t scratch_bytes, const DtFusion* dtf, bool flags_zeroed) {
    const RowStrides dense{0, 0, 0};
    if (!rs) rs = &dense;
    if (dtf && !dt_fusable(a, *dtf)) return cudaErrorInvalidValue;
    const bool bdl = a.layout == SACC_LAYOUT_BDL;
    const unsigned long long cw = a.c_width, B = a.batch, D = a.channels, L = a.length, G = a.groups;
    const CUtensorMapDataType dt = a.dtype == SACC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap tu{}, td{}, tz{}, tb{}, tc{}, ty{};
    bool ok;
    if (bdl) {
        const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_64B;
        ok = make_map_2d(&tu, dt, a.u, L, B * D, L * 2, kT, kLanes, sw) &&
             make_map_2d(&td, dt, a.delta, L, B * D, L * 2, kT, kLanes, sw) &&
             make_map_2d(&tz, dt, a.z ? a.z : a.u, L, B * D, L * 2, kT, kLanes, sw) &&
             make_map_2d(&ty, dt, a.y, L, B * D, L * 2, kT, kLanes, sw) &&
             make_map_2d(&tb, dt, a.b, L, B * G * kN, L * 2, kT, kN, CU_TENSOR_MAP_SWIZZLE_NONE) &&
             make_map_2d(&tc, dt, a.c, L, B * G * cw, L * 2, kT, static_cast<unsigned>(cw), CU_TENSOR_MAP_SWIZZLE_NONE);
    } else {
        ok = make_map_3d(&tu, dt, a.u, D, L, B, kLanes, kT) &&
             (dtf ? make_map_3d(&td, dt, dtf->dt, static_cast<unsigned long long>(dtf->rank), L, B,
                                static_cast<unsigned>(dtf->rank), kT, dtf->ld)
                  : make_map_3d(&td, dt, a.delta, D, L, B, kLanes, kT)) &&
             make_map_3d(&tz, dt, a.z ? a.z : a.u, D, L, B, kLanes, kT / 2, a.z ? rs->z : 0) &&
             make_map_3d(&ty, dt, a.y, D, L, B, kLanes, kT) && make_map_3d(&tb, dt, a.b, G * kN, L, B, kN, kT, rs->b) &&
             make_map_3d(&tc, dt, a.c, G * cw, L, B, static_cast<unsigned>(cw), kT, rs->c);
    }
    if (!ok) return cudaErrorInvalidValue; // tensor-map encoding refused the (checked) layout
    BulkParams p{};
    p.a = a.a; p.d = a.d; p.bias = a.delta_bias; p.h0 = a.h0; p.h_final = a.h_final;
    p.length = L; p.channels = D; p.per_group = D / G; p.groups = static_cast<unsigned>(G);
    p.a_shared = a.a_rows == 1; p.c_full = cw != 1; p.has_d = a.d != nullptr; p.softplus = a.delta_softplus != 0;
    p.nchunks = static_cast<int>((L + kT - 1) / kT);
    p.cu = bdl ? nullptr : a.cu_seqlens;
    p.y = a.y;
    p.zg = a.z;
    p.zld = rs->z ? rs->z : D;
    p.wdt = dtf ? dtf->w : nullptr;
    const unsigned long long rows = a.cu_seqlens ? static_cast<unsigned long long>(a.nseq) : B; // sequences
    p.units = rows * (D / kLanes);
    p.parts = 1;
    p.epoch = 0;
    const Pick loop = pick_for(a, dtf, 1);
    cudaError_t attr = loop.prepare();
    if (attr != cudaSuccess) return attr;
    const unsigned long long wave = resident_ctas(loop);
    void* args[] = {&tu, &td, &tz, &tb, &tc, &ty, &p};
    // Packed varlen sequences (one CTA per sequence x 128 channels: persistent
    // CTAs were slower, each sequence's start waiting on its h0 row) and
    // launches that fit one wave or gain nothing from a split: one item per CTA.
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    p.passes = 1;
    if (scratch != nullptr) {
        Pick fk{};
        const int fused = fused_plan(a, dtf, fk);
        if (fused && scratch_bytes >= fused_scratch_bytes(p.units, fused) &&
            (reinterpret_cast<std::uintptr_t>(scratch) & 15u) == 0) {
            // Few units over long sequences, with scratch: every part's local
            // pass, hand-off and final pass in one cooperative launch (every
            // CTA resident: a part waits on the flags of the parts before it).
            p.parts = fused;
            p.passes = 2;
            p.scratch = static_cast<float*>(scratch);
            p.epoch = next_epoch();
            // The flags stay in the scratch after the launch (nothing in it
            // overwrites them), and a CUDA graph replays this launch with the
            // same epoch: they must be zero when it starts, so that a part
            // never sees a flag that an earlier launch or replay left (the
            // epoch is never zero).  The block pipeline's conv kernel clears
            // them; other callers get a memset here.
            if (!flags_zeroed) {
                const std::size_t records = static_cast<std::size_t>(p.units) * fused * (kN + 1) * kLanes;
                const cudaError_t me = cudaMemsetAsync(p.scratch + records, 0, static_cast<std::size_t>(p.units) * fused * 8, stream);
                if (me != cudaSuccess) return me;
            }
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(static_cast<unsigned>(p.units * fused));
            cfg.blockDim = dim3(static_cast<unsigned>(fk.threads));
            cfg.dynamicSmemBytes = fk.smem;
            cfg.stream = stream;
            cudaLaunchAttribute attrs[2]{};
            attrs[0].id = cudaLaunchAttributeCooperative;
            attrs[0].val.cooperative = 1;
            cfg.attrs = attrs;
            cfg.numAttrs = 1;
            return cudaLaunchKernelExC(&cfg, fk.fn, args);
        }
    }
    if (bdl && a.z) {
        // The walks below take the (B, D, L) gate as two 16-token halves per
        // chunk: an unswizzled map with a 16 x 128 box.
        if (!make_map_2d(&tz, dt, a.z, L, B * D, L * 2, kT / 2, kLanes, CU_TENSOR_MAP_SWIZZLE_NONE)) return cudaErrorInvalidValue;
    }
    const int chunked = p.cu ? 0 : chunk_parts(p.units, static_cast<unsigned long long>(sms), p.nchunks, L);
    if (chunked) {
        // Few units over long sequences: the chunk-parallel passes (stream
        // ordered, no workspace: the hand-offs live in y like the split's).
        const Pick one = pick_for(a, dtf, 0);
        if ((attr = one.prepare()) != cudaSuccess) return attr;
        p.parts = chunked;
        p.phase = 1;
        cudaError_t e = launch_pdl(one.fn, dim3(static_cast<unsigned>(p.units * chunked)), dim3(kLanes), one.smem, stream, args);
        if (e != cudaSuccess) return e;
        const unsigned long long threads = rows * D;
        const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
        if (a.dtype == SACC_DTYPE_BF16)
            e = bdl ? launch_pdl_k(combine_kernel<__nv_bfloat16, true>, dim3(blocks), dim3(256), 0, stream, p, rows)
                    : launch_pdl_k(combine_kernel<__nv_bfloat16, false>, dim3(blocks), dim3(256), 0, stream, p, rows);
        else
            e = bdl ? launch_pdl_k(combine_kernel<__half, true>, dim3(blocks), dim3(256), 0, stream, p, rows)
                    : launch_pdl_k(combine_kernel<__half, false>, dim3(blocks), dim3(256), 0, stream, p, rows);
        if (e != cudaSuccess) return e;
        p.phase = 2;
        p.item0 = p.units;
        return launch_pdl(one.fn, dim3(static_cast<unsigned>(p.units * (chunked - 1))), dim3(kLanes), one.smem, stream, args);
    }
    if (quad_eligible(a) && p.units <= 2ull * static_cast<unsigned long long>(sms)) {
        // Few units (at most two CTAs per SM): four threads per lane.
        const Pick qk = pick_quad(a, dtf, 0);
        if ((attr = qk.prepare()) != cudaSuccess) return attr;
        return launch_pdl(qk.fn, dim3(static_cast<unsigned>(p.units)), dim3(kLanes * kQ), qk.smem, stream, args);
    }
    const Pick one = pick_for(a, dtf, 0);
    if ((attr = one.prepare()) != cudaSuccess) return attr;
    const unsigned long long wave0 = resident_ctas(one);
    if (p.cu || (p.units <= wave0 && (5 * p.units <= 3 * wave0 || p.nchunks < 4))) {
        // One wave (or packed sequences): one CTA per unit.
        return launch_pdl(one.fn, dim3(static_cast<unsigned>(p.units)), dim3(kLanes), one.smem, stream, args);
    }
    // More units than 60 % of one wave: (unit, part) items, part-major, one
    // per CTA of a plain multi-wave grid (a one-wave launch that fills most
    // slots ends on the SMs' slowest CTAs: at 512 units for 592 slots the
    // split was 5-8 % faster, at 320 units within +-5 %).  Part k of a unit
    // waits on part k - 1's hand-off, which has a lower block index and so
    // was dispatched first; the wait is bounded (a fault, never a hang).
    p.parts = split_parts(p.units, wave, p.nchunks, L);
    if (p.parts > 1) p.epoch = next_epoch();
    return launch_pdl(loop.fn, dim3(static_cast<unsigned>(p.units * static_cast<unsigned long long>(p.parts))), dim3(kLanes),
                      loop.smem, stream, args);
}

cudaError_t load_scan_bulk_kernels(std::string& report) {
    const char* names[2] = {"bld", "bdl"};
    for (int dtype : {SACC_DTYPE_BF16, SACC_DTYPE_F16})
        for (int bdl = 0; bdl < 2; ++bdl)
            for (int z = 0; z < 4; ++z) {
                if (!bdl && (z & 2) == 0) continue; // (B, L, D) always has a full-width C
                const Pick k = pick(dtype, bdl != 0, (z & 1) != 0, (z & 2) != 0, false);
                const Pick kl = pick(dtype, bdl != 0, (z & 1) != 0, (z & 2) != 0, true);
                cudaFuncAttributes attr{}, attr_loop{};
                cudaError_t e = cudaFuncGetAttributes(&attr, k.fn);
                if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr_loop, kl.fn);
                if (e == cudaSuccess) e = k.prepare();
                if (e == cudaSuccess) e = kl.prepare();
                if (e != cudaSuccess) return e;
                report += std::string("kernel=scan_bulk_") + names[bdl] + (dtype == SACC_DTYPE_BF16 ? "_bf16" : "_f16") +
                          ((z & 1) ? "_gate" : "") + ((z & 2) ? "" : "_rank1c") + " registers=" + std::to_string(attr.numRegs) +
                          " local_bytes=" + std::to_string(attr.localSizeBytes) +
                          " dynamic_shared_bytes=" + std::to_string(k.smem) + "\n";
            }
    return cudaSuccess;
}

cudaError_t launch_wait_probe(std::uint32_t limit, cudaStream_t stream) {
    wait_probe_kernel<<<1, 32, 0, stream>>>(limit);
    return cudaGetLastError();
}

cudaError_t read_bulk_fault(unsigned* out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_bulk_fault, sizeof(unsigned));
    if (e != cudaSuccess || !clear) return e;
    const unsigned zero = 0;
    return cudaMemcpyToSymbol(g_bulk_fault, &zero, sizeof(unsigned));
}

} // namespace sacc
