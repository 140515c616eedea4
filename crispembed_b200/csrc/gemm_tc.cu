// gemm_tc.cu -- grouped GEMM over block-quantized weights on tcgen05 / TMEM.
//
// Replaces the ggml_mul_mat / ggml_mul_mat_id products of the encoder graph
// (src/crispembed.cpp:1160-1177, :1320, :1333-1371, :1411-1416 of the
// reference), computing for every group g (expert, or one group for a dense
// layer) and every activation row r in the group's row range:
//
//     out[r, n] = epilogue( sum_k W_g[n, k] * X[r, k] )
//
// Operands (tcgen05.mma kind::f16, both from shared memory, 128-byte swizzle):
//   A = weight tile, 128 output features x 64 k, dequantized by eight warps from
//       the Q8_0 / Q4_K / fp16 planes in global memory and written to shared
//       memory in the MMA's swizzled K-major layout;
//   B = activation tile, up to 256 rows x 64 k fp16, loaded by TMA;
//   D = fp32 accumulator in TMEM, [128 features (lanes)] x [256 rows (columns)],
//       double buffered (all 512 TMEM columns) so the epilogue of one tile
//       overlaps the next tile.  An M=128,K=16 MMA costs the same time for any
//       N <= 256, hence the full-width 256-row tile.
//
// Warp roles (640 threads, one persistent CTA per SM):
//   warp 0        TMA producer of activation stages
//   warp 1        TMEM owner + single-thread MMA issuer
//   warps 4..11   dequant producers, two warpgroups taking alternate K-blocks
//                 (thread i of a warpgroup <-> weight row i of the tile)
//   warps 12..19  epilogue, two warpgroups taking alternate 32-row chunks
//                 (thread i <-> output feature i): bias, GELU, then each warp
//                 stages its 32x32 block in shared memory for one TMA store
//                 (rows past a group's end are stored directly instead, so a
//                 tile never writes into the next expert's rows)
// Tiles (group, token tile, feature tile) are distributed round-robin; the
// group table is read from device memory, so no host synchronisation is
// needed between routing and the expert GEMMs.
//
// The description above is the single-CTA kernel (ceb_gemm_kernel: other
// widths).  Layers whose width is a multiple of 256 run ceb_gemm_pair_kernel
// further down: CTA pairs with tokens as the MMA's M (256 per pair) and 256
// features as N.  Its weights are usually fp16 planes expanded once at load
// (ceb_wplane_expand_f16), which both CTAs TMA-load straight into the operand
// stage; quantized planes are dequantized in shared memory as here.
#include <cstdio>
#include <cstdlib>

#include "ceb_internal.h"
#include "common.cuh"

namespace {

constexpr int BM = 128;
constexpr int BN = 256;               // activation rows (tokens) per tile = max MMA N
constexpr int BK = 64;
#ifndef CEB_GEMM_S
#define CEB_GEMM_S 3
#endif
#ifndef CEB_GEMM_R
#define CEB_GEMM_R 4
#endif
constexpr int S = CEB_GEMM_S;         // pipeline stages (A + B tiles)
constexpr int R = CEB_GEMM_R;         // raw (still quantized) weight stages
constexpr int RAW_STAGE = 8704;       // largest quantized block (Q8_0)
constexpr int MAXG = 64;
constexpr int A_STAGE_BYTES = BM * BK * 2;   // 16 KB, written by the dequant warps
constexpr int B_STAGE_BYTES = BN * BK * 2;   // 32 KB, written by TMA
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr uint32_t TMEM_COLS = 512;          // two BN-column fp32 accumulators
constexpr int DEQ_WG = 2, EPI_WG = 2;
constexpr int DEQ_WARP0 = 4, EPI_WARP0 = DEQ_WARP0 + 4 * DEQ_WG;
constexpr int NTHREADS = 32 * (EPI_WARP0 + 4 * EPI_WG);
#ifndef CEB_GEMM_TMA_STORE
#define CEB_GEMM_TMA_STORE 1
#endif
constexpr int STAGING_SLOT = 32 * 32 * 4;    // one 32x32 fp32 output block per slot
constexpr int STAGING_BYTES = CEB_GEMM_TMA_STORE ? 4 * EPI_WG * STAGING_SLOT : 0;  // one slot per epilogue warp
static_assert(2 * BN <= (int)TMEM_COLS, "TMEM budget");

// The dequant warpgroups take alternate K-blocks. Every raw stage must always be
// consumed by the same warpgroup: with an odd ring a stage's items alternate
// between warpgroups, one of them can wait on a phase two ahead of the barrier,
// and the mbarrier's parity test then passes on a stale phase.
static_assert(R % DEQ_WG == 0, "raw stages must map to one dequant warpgroup each");
constexpr int NBARS = 2 * S + 4 + 1 + 2 * R;
constexpr size_t SMEM_BYTES = 1024 /*align slack*/ + (size_t)S * STAGE_BYTES + (size_t)R * RAW_STAGE + STAGING_BYTES +
                              NBARS * 8 + 16 + 3 * (MAXG + 1) * 4;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");

struct Shared {
    uint64_t* bars;
    uint32_t* tmem_slot;
    int* abort;
    int* g_tile;
    int* g_row;
    int* g_cnt;
    uint8_t* stages;   // stage s: A at s*STAGE_BYTES, B right after
    uint8_t* raw;      // raw weight stages
    uint8_t* staging;  // epilogue output blocks
};

CEB_DEV Shared carve(uint8_t* raw) {
    Shared s;
    uintptr_t p = (reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023);
    s.stages = reinterpret_cast<uint8_t*>(p);
    p += (size_t)S * STAGE_BYTES;
    s.raw = reinterpret_cast<uint8_t*>(p);
    p += (size_t)R * RAW_STAGE;
    s.staging = reinterpret_cast<uint8_t*>(p);
    p += STAGING_BYTES;
    s.bars = reinterpret_cast<uint64_t*>(p);
    p += NBARS * 8;
    s.tmem_slot = reinterpret_cast<uint32_t*>(p);
    s.abort = reinterpret_cast<int*>(p + 4);
    p += 16;
    s.g_tile = reinterpret_cast<int*>(p);
    s.g_row = s.g_tile + (MAXG + 1);
    s.g_cnt = s.g_row + (MAXG + 1);
    return s;
}

// barrier indices
CEB_DEV int BAR_FULL(int s) { return s; }       // TMA bytes + one arrive per dequant warp
CEB_DEV int BAR_EMPTY(int s) { return S + s; }  // MMA commit
CEB_DEV int BAR_ACC_FULL(int b) { return 2 * S + b; }
CEB_DEV int BAR_ACC_EMPTY(int b) { return 2 * S + 2 + b; }
CEB_DEV int BAR_DRAIN() { return 2 * S + 4; }
CEB_DEV int BAR_RAW_FULL(int r) { return 2 * S + 5 + r; }      // bulk-copy bytes
CEB_DEV int BAR_RAW_EMPTY(int r) { return 2 * S + 5 + R + r; } // one arrive per dequant warp

struct TileInfo {
    int g, ft, row0, rows;
};

CEB_DEV TileInfo decode_tile(const Shared& S_, int G, int n_ftiles, int t) {
    int g = 0;
    while (g + 1 < G && t >= S_.g_tile[g + 1]) ++g;
    int local = t - S_.g_tile[g];
    TileInfo ti;
    ti.g = g;
    ti.ft = local % n_ftiles;
    int tt = local / n_ftiles;
    ti.row0 = S_.g_row[g] + tt * BN;
    int rem = S_.g_cnt[g] - tt * BN;
    ti.rows = rem < BN ? rem : BN;
    return ti;
}

// ---- raw weight fragments held in registers while in flight -------------
template <int FMT>
struct Raw;
template <>
struct Raw<CEB_W_Q8_0> {
    uint4 q[4];
    uint32_t sc;
};
template <>
struct Raw<CEB_W_Q4_K> {
    uint4 q[2];
    uint4 s;
};
template <>
struct Raw<CEB_W_F16> {
    uint4 q[8];
};

// Row r's share of a raw block in shared memory (layouts in ceb_internal.h).
template <int FMT>
CEB_DEV void load_raw_smem(const uint8_t* blk, int r, Raw<FMT>& out);

template <>
CEB_DEV void load_raw_smem<CEB_W_Q8_0>(const uint8_t* blk, int r, Raw<CEB_W_Q8_0>& o) {
#pragma unroll
    for (int c = 0; c < 4; ++c) o.q[c] = *reinterpret_cast<const uint4*>(blk + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
    o.sc = *reinterpret_cast<const uint32_t*>(blk + 8192 + 4 * r);
}
template <>
CEB_DEV void load_raw_smem<CEB_W_Q4_K>(const uint8_t* blk, int r, Raw<CEB_W_Q4_K>& o) {
#pragma unroll
    for (int c = 0; c < 2; ++c) o.q[c] = *reinterpret_cast<const uint4*>(blk + r * 32 + ((c ^ ((r >> 2) & 1)) << 4));
    o.s = *reinterpret_cast<const uint4*>(blk + 4096 + 16 * r);
}
template <>
CEB_DEV void load_raw_smem<CEB_W_F16>(const uint8_t*, int, Raw<CEB_W_F16>&) {}

// ---- conversion to fp16 pairs: word c holds k = 2c (low half), 2c+1
template <int FMT>
CEB_DEV void convert(const Raw<FMT>& r, uint32_t (&o)[32]);

template <>
CEB_DEV void convert<CEB_W_Q8_0>(const Raw<CEB_W_Q8_0>& r, uint32_t (&o)[32]) {
    const __half2 d0 = __half2half2(__ushort_as_half((unsigned short)(r.sc & 0xFFFF)));
    const __half2 d1 = __half2half2(__ushort_as_half((unsigned short)(r.sc >> 16)));
    const uint32_t* wd = reinterpret_cast<const uint32_t*>(r.q);
#pragma unroll
    for (int w = 0; w < 16; ++w) i8x4_to_h2x2(wd[w], w < 8 ? d0 : d1, o[2 * w], o[2 * w + 1]);
}

CEB_DEV float nib_f(uint32_t v, int byte) {
    return __uint_as_float(0x4B000000u | ((v >> (8 * byte)) & 0xFFu)) - 8388608.0f;
}

template <>
CEB_DEV void convert<CEB_W_Q4_K>(const Raw<CEB_W_Q4_K>& r, uint32_t (&o)[32]) {
    const float dA = __uint_as_float(r.s.x), mA = __uint_as_float(r.s.y);
    const float dB = __uint_as_float(r.s.z), mB = __uint_as_float(r.s.w);
    const uint32_t* wd = reinterpret_cast<const uint32_t*>(r.q);
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        const uint32_t lo = wd[w] & 0x0F0F0F0Fu, hi = (wd[w] >> 4) & 0x0F0F0F0Fu;
        float a0 = __fsub_rn(__fmul_rn(dA, nib_f(lo, 0)), mA), a1 = __fsub_rn(__fmul_rn(dA, nib_f(lo, 1)), mA);
        float a2 = __fsub_rn(__fmul_rn(dA, nib_f(lo, 2)), mA), a3 = __fsub_rn(__fmul_rn(dA, nib_f(lo, 3)), mA);
        float b0 = __fsub_rn(__fmul_rn(dB, nib_f(hi, 0)), mB), b1 = __fsub_rn(__fmul_rn(dB, nib_f(hi, 1)), mB);
        float b2 = __fsub_rn(__fmul_rn(dB, nib_f(hi, 2)), mB), b3 = __fsub_rn(__fmul_rn(dB, nib_f(hi, 3)), mB);
        o[2 * w] = h2_as_u32(__floats2half2_rn(a0, a1));
        o[2 * w + 1] = h2_as_u32(__floats2half2_rn(a2, a3));
        o[16 + 2 * w] = h2_as_u32(__floats2half2_rn(b0, b1));
        o[17 + 2 * w] = h2_as_u32(__floats2half2_rn(b2, b3));
    }
}

template <>
CEB_DEV void convert<CEB_W_F16>(const Raw<CEB_W_F16>& r, uint32_t (&o)[32]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        o[4 * i] = r.q[i].x;
        o[4 * i + 1] = r.q[i].y;
        o[4 * i + 2] = r.q[i].z;
        o[4 * i + 3] = r.q[i].w;
    }
}

// erf-GELU 0.5 x (1 + erf(x / sqrt 2)) with erf from Abramowitz & Stegun 7.1.26
// (|error| <= 1.5e-7 on erf), far below the fp16/fp32 rounding of the output:
//   z = |x|/sqrt2, t = 1/(1 + p z), erf(z) = 1 - t(a1 + t(a2 + t(a3 + t(a4 + t a5)))) exp(-z^2).
// The reciprocal and the exponential use the MUFU approximations (rel. error ~2^-22),
// exp(-z^2) as 2^(-(z sqrt(log2 e))^2) with the scaling folded into one constant.
CEB_DEV float rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
CEB_DEV float ex2_approx(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
CEB_DEV float gelu_as(float x) {
    constexpr float kZ = 0.70710678118654752f;             // 1/sqrt(2)
    constexpr float kE = 0.84932180028801904f;             // sqrt(log2 e) / sqrt(2)
    const float ax = fabsf(x);
    const float t = rcp_approx(fmaf(0.3275911f * kZ, ax, 1.0f));
    float p = fmaf(1.061405429f, t, -1.453152027f);
    p = fmaf(p, t, 1.421413741f);
    p = fmaf(p, t, -0.284496736f);
    p = fmaf(p, t, 0.254829592f);
    const float u = ax * kE;
    const float e = ex2_approx(-u * u);                     // exp(-x^2/2)
    const float erf_abs = fmaf(-p * t, e, 1.0f);            // erf(|x|/sqrt2)
    const float h = 0.5f * x;
    return fmaf(fabsf(h), erf_abs, h);                      // 0.5x + 0.5|x| erf(|x|/sqrt2)
}
// gelu_as on two values with packed fp32 arithmetic: the same operations in the same
// order, so both results equal gelu_as's bit for bit. The polynomial is evaluated with
// negated coefficients (Horner with round-to-nearest is odd in them), which yields
// -p t without a separate negation; (x kE)^2 = (|x| kE)^2 exactly.
CEB_DEV f32x2 gelu_as2(f32x2 x) {
    constexpr float kZ = 0.70710678118654752f;
    constexpr float kE = 0.84932180028801904f;
    float x0, x1;
    f2_unpack(x, x0, x1);
    const f32x2 ax = f2_pack(fabsf(x0), fabsf(x1));
    f32x2 t = f2_fma(f2_splat(0.3275911f * kZ), ax, f2_splat(1.0f));
    {
        float t0, t1;
        f2_unpack(t, t0, t1);
        t = f2_pack(rcp_approx(t0), rcp_approx(t1));
    }
    f32x2 p = f2_fma(f2_splat(-1.061405429f), t, f2_splat(1.453152027f));
    p = f2_fma(p, t, f2_splat(-1.421413741f));
    p = f2_fma(p, t, f2_splat(0.284496736f));
    p = f2_fma(p, t, f2_splat(-0.254829592f));  // -p of gelu_as
    const f32x2 u = f2_mul(x, f2_splat(kE));
    const f32x2 s = f2_mul(u, u);
    float s0, s1;
    f2_unpack(s, s0, s1);
    const f32x2 e = f2_pack(ex2_approx(-s0), ex2_approx(-s1));
    const f32x2 erf_abs = f2_fma(f2_mul(p, t), e, f2_splat(1.0f));
    const f32x2 h = f2_mul(x, f2_splat(0.5f));
    return f2_fma(f2_mul(ax, f2_splat(0.5f)), erf_abs, h);
}

template <int FMT>
__global__ void __launch_bounds__(NTHREADS, 1)
    ceb_gemm_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap omap,
                    const ceb_wplane w, const ceb_gemm_args a) {
    extern __shared__ uint8_t smem_raw[];
    const Shared SH = carve(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = a.offsets ? w.n_groups : 1;
    const int n_ftiles = w.n_out / BM;
    const int nkb = w.k / BK;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NBARS; ++i) {
            uint32_t cnt = 1;
            if (i < S) cnt = FMT == CEB_W_F16 ? 1 : 1 + 4;              // stage full: TMA (+ 4 dequant warps)
            if (i >= 2 * S + 5 + R && i < 2 * S + 5 + 2 * R) cnt = 4;  // raw empty: one dequant warpgroup
            if (i >= 2 * S + 2 && i < 2 * S + 4) cnt = 4 * EPI_WG;      // acc empty: epilogue warps
            mbar_init(smem_u32(&SH.bars[i]), cnt);
        }
        fence_mbar_init();
        *SH.abort = 0;
        int tiles = 0;
        for (int g = 0; g < G; ++g) {
            int r0 = a.offsets ? a.offsets[g] : 0;
            int r1 = a.offsets ? a.offsets[g + 1] : a.m_rows;
            if (r0 < 0 || r1 < r0 || r1 > a.m_rows) {
                if (a.err) atomicCAS(a.err, 0, (int)CEB_DEVERR_BAD_GROUP);
                r0 = r1 = 0;
            }
            SH.g_tile[g] = tiles;
            SH.g_row[g] = r0;
            SH.g_cnt[g] = r1 - r0;
            tiles += ((r1 - r0 + BN - 1) / BN) * n_ftiles;
        }
        SH.g_tile[G] = tiles;
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmap);
        tma_prefetch_desc(&omap);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(SH.tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *SH.tmem_slot;
    const int total = SH.g_tile[G];
    volatile int* abort = SH.abort;
    auto bar = [&](int i) { return smem_u32(&SH.bars[i]); };
    // bounded barrier wait; a timeout records its site as code | (barrier index + 1) << 16
    auto wait_at = [&](int i, uint32_t parity, int code) {
        return mbar_wait(bar(i), parity, abort, a.err, code | ((i + 1) << 16));
    };
    auto a_stage = [&](int s) { return SH.stages + (size_t)s * STAGE_BYTES; };
    auto b_stage = [&](int s) { return SH.stages + (size_t)s * STAGE_BYTES + A_STAGE_BYTES; };
    auto wblock = [&](const TileInfo& ti, int kb) {
        return w.q + (((size_t)ti.g * n_ftiles + ti.ft) * nkb + kb) * (size_t)w.blk_bytes;
    };

    if (warp == 0) {
        // ------------------------------------------------ TMA producer (activation tiles)
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                const TileInfo ti = decode_tile(SH, G, n_ftiles, t);
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % S;
                    if (!wait_at(BAR_EMPTY(s), ((it / S) & 1) ^ 1, CEB_DEVERR_TIMEOUT_TMA)) {
                        ok = false;
                        break;
                    }
                    if (FMT == CEB_W_F16) {  // fp16 weights are stored as the swizzled A image
                        mbar_arrive_expect_tx(bar(BAR_FULL(s)), B_STAGE_BYTES + A_STAGE_BYTES);
                        bulk_load(smem_u32(a_stage(s)), wblock(ti, kb), A_STAGE_BYTES, bar(BAR_FULL(s)));
                    } else {
                        mbar_arrive_expect_tx(bar(BAR_FULL(s)), B_STAGE_BYTES);
                    }
                    tma_load_2d(smem_u32(b_stage(s)), &tmap, bar(BAR_FULL(s)), kb * BK, ti.row0);
                }
            }
            if (!ok) {  // let issued copies land before the CTA can exit
                const uint32_t n = it < S ? it : S;
                for (uint32_t i = it - n; i < it; ++i) mbar_wait(bar(BAR_FULL(i % S)), (i / S) & 1, nullptr, nullptr, 0);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t it = 0, lt = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++lt) {
                const TileInfo ti = decode_tile(SH, G, n_ftiles, t);
                const int ab = lt & 1;
                if (!wait_at(BAR_ACC_EMPTY(ab), ((lt >> 1) & 1) ^ 1, CEB_DEVERR_TIMEOUT_MMA)) break;
                tc_fence_after();
                int n = (ti.rows + 15) & ~15;
                n = n < 16 ? 16 : n;
                const uint32_t idesc = idesc_f16_f32(BM, n);
                const uint32_t d_tmem = tmem + (uint32_t)(ab * BN);
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % S;
                    if (!wait_at(BAR_FULL(s), (it / S) & 1, CEB_DEVERR_TIMEOUT_MMA)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t adesc = smem_desc_sw128(smem_u32(a_stage(s)));
                    const uint64_t bdesc = smem_desc_sw128(smem_u32(b_stage(s)));
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        mma_f16_ss(d_tmem, adesc + (uint64_t)(kk * 2), bdesc + (uint64_t)(kk * 2), idesc,
                                   (kb | kk) != 0);
                    mma_commit(bar(BAR_EMPTY(s)));
                }
                if (ok) mma_commit(bar(BAR_ACC_FULL(ab)));
            }
            // every issued MMA has retired before TMEM can be released
            mma_commit(bar(BAR_DRAIN()));
            mbar_wait(bar(BAR_DRAIN()), 0, nullptr, nullptr, 0);
        }
    } else if (warp == 2) {
        // ------------------------------------------------ weight loader (quantized blocks -> raw stages)
        if (FMT != CEB_W_F16 && lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                const TileInfo ti = decode_tile(SH, G, n_ftiles, t);
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int rs = it % R;
                    if (!wait_at(BAR_RAW_EMPTY(rs), ((it / R) & 1) ^ 1, CEB_DEVERR_TIMEOUT_TMA)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(bar(BAR_RAW_FULL(rs)), (uint32_t)w.blk_bytes);
                    bulk_load(smem_u32(SH.raw + (size_t)rs * RAW_STAGE), wblock(ti, kb), (uint32_t)w.blk_bytes,
                              bar(BAR_RAW_FULL(rs)));
                }
            }
            if (!ok) {  // let issued copies land before the CTA can exit
                const uint32_t n = it < R ? it : R;
                for (uint32_t i = it - n; i < it; ++i)
                    mbar_wait(bar(BAR_RAW_FULL(i % R)), (i / R) & 1, nullptr, nullptr, 0);
            }
        }
    } else if (warp >= DEQ_WARP0 && warp < EPI_WARP0) {
        // ------------------------------------------------ dequant (raw stage -> fp16 A stage)
        if (FMT != CEB_W_F16) {
            const int wg = (warp - DEQ_WARP0) >> 2;  // this warpgroup takes items i with i % DEQ_WG == wg
            const int r = 32 * (warp & 3) + lane;    // weight row within the tile
            const int my_tiles = blockIdx.x < total ? (total - 1 - blockIdx.x) / gridDim.x + 1 : 0;
            const int n_items = my_tiles * nkb;
            for (int i = wg; i < n_items; i += DEQ_WG) {
                const int rs = i % R, s = i % S;
                if (!__all_sync(0xffffffffu, wait_at(BAR_RAW_FULL(rs), (i / R) & 1, CEB_DEVERR_TIMEOUT_DEQ)))
                    break;
                Raw<FMT> raw;
                load_raw_smem<FMT>(SH.raw + (size_t)rs * RAW_STAGE, r, raw);
                uint32_t o[32];
                convert<FMT>(raw, o);  // consumes the loaded values: the raw stage may be refilled now
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(BAR_RAW_EMPTY(rs)));
                if (!__all_sync(0xffffffffu, wait_at(BAR_EMPTY(s), ((i / S) & 1) ^ 1, CEB_DEVERR_TIMEOUT_DEQ)))
                    break;
                // 128-byte swizzled K-major row: 16-byte chunk c lands at chunk c ^ (row & 7)
                uint8_t* row = a_stage(s) + r * 128;
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) =
                        make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(BAR_FULL(s)));
            }
        }
    } else if (warp >= EPI_WARP0) {
        // ------------------------------------------------ epilogue
        const int ew = warp - EPI_WARP0;
        const int wg = ew >> 2;                  // this warpgroup takes 32-column chunks c with c % EPI_WG == wg
        const int q = warp & 3;                  // features 32q .. 32q+31 of the tile (TMEM lanes)
        const uint32_t lane_addr = (uint32_t)(32 * q) << 16;
        const bool f16 = (a.epi & CEB_EPI_F16_OUT) != 0, gelu = (a.epi & CEB_EPI_GELU) != 0;
        const int esz = f16 ? 2 : 4;
        uint8_t* slot = SH.staging + (size_t)ew * STAGING_SLOT;
        uint32_t lt = 0, nstore = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, ++lt) {
            const TileInfo ti = decode_tile(SH, G, n_ftiles, t);
            const int ab = lt & 1;
            if (!__all_sync(0xffffffffu,
                            wait_at(BAR_ACC_FULL(ab), (lt >> 1) & 1, CEB_DEVERR_TIMEOUT_EPI)))
                break;
            tc_fence_after();
            const int n0 = ti.ft * BM + 32 * q;
            const int n = n0 + lane;
            const float bv = (a.epi & CEB_EPI_BIAS) ? a.bias[(size_t)ti.g * a.bias_group_stride + n] : 0.0f;
            for (int c0 = 32 * wg; c0 < ti.rows; c0 += 32 * EPI_WG) {
                uint32_t v[32];
                tmem_ld32(tmem + lane_addr + (uint32_t)(ab * BN + c0), v);
                tmem_ld_wait();
                float x[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    x[j] = __uint_as_float(v[j]) + bv;
                    if (gelu) x[j] = gelu_as(x[j]);
                }
                const int lim = ti.rows - c0;
                if (CEB_GEMM_TMA_STORE && lim >= 32) {
                    // full 32-row block: stage [row][feature] in shared memory, one TMA store
                    if (nstore >= 1) {  // the previous store has finished reading the slot
                        if (lane == 0) bulk_wait_read<0>();
                        __syncwarp();
                    }
                    if (f16) {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            reinterpret_cast<__half*>(slot)[j * 32 + lane] = __float2half_rn(x[j]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) reinterpret_cast<float*>(slot)[j * 32 + lane] = x[j];
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&omap, smem_u32(slot), n0, ti.row0 + c0);
                        bulk_commit();
                    }
                    ++nstore;
                } else if (f16) {
                    __half* o = reinterpret_cast<__half*>(a.out) + (size_t)(ti.row0 + c0) * a.ldo + n;
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (j < lim) o[(size_t)j * a.ldo] = __float2half_rn(x[j]);
                } else {
                    float* o = reinterpret_cast<float*>(a.out) + (size_t)(ti.row0 + c0) * a.ldo + n;
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (j < lim) o[(size_t)j * a.ldo] = x[j];
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(BAR_ACC_EMPTY(ab)));
        }
        (void)esz;
        if (lane == 0) bulk_wait<0>();  // output stores complete before the CTA retires
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

template <int FMT>
int launch_fmt(const CUtensorMap& map, const CUtensorMap& omap, const ceb_wplane& w, const ceb_gemm_args& a, int grid,
               cudaStream_t st) {
    if (int rc = ceb_func_smem(reinterpret_cast<const void*>(ceb_gemm_kernel<FMT>), SMEM_BYTES)) return rc;
    ceb_gemm_kernel<FMT><<<grid, NTHREADS, SMEM_BYTES, st>>>(map, omap, w, a);
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}


// ===========================================================================
// CTA-pair kernel (cluster of 2, tcgen05.mma.cta_group::2, M = 256).
//
// Orientation: tokens are the MMA's M (A = activations, 128 rows per CTA, TMA),
// features are N (B = dequantized weights, 128 rows per CTA, N = 256 per pair).
// Each CTA's tensor memory holds D for its 128 tokens x all 256 features of the
// pair tile, double buffered (2 x 256 columns).  Per SM and K-block this moves
// half the shared-memory bytes of the 1-CTA kernel for the activations and
// runs the tensor pipe at its full rate (one M=256,N=256,K=16 MMA per 128
// cycles per pair, measured), against ~178 cycles per M=128 MMA on one SM.
//
// Barriers: FULL[s] lives in the leader (rank 0): the leader's TMA thread posts
// the expected bytes of both CTAs' activation tiles, both CTAs' TMA loads count
// their bytes on it, and the leader's 4 dequant warps arrive on it.  Rank 1's
// dequant warps arrive on its local W_FULL[s]; a relay thread of rank 1 then
// copies 16 bytes into the leader's shared memory with cp.async.bulk, whose
// complete_tx lands on FULL[s] (the leader expects 2 activation tiles + 16 B).
// The leader's MMA commits EMPTY[s] / ACC_FULL[b] to both CTAs.  ACC_EMPTY[b]
// takes the leader's epilogue warps plus 16 relayed bytes once rank 1's
// epilogue warps have arrived on its local ACC_FREE[b].  The cross-CTA signals
// are asynchronous copies: a blocking cluster-scope release arrive costs ~1500
// cycles per call, three times the MMA time of a K-block.
namespace pair {
constexpr int TOK = 128;                     // tokens per CTA
constexpr int FEAT = 256;                    // features per pair tile (MMA N)
constexpr int X_BYTES = TOK * BK * 2;        // 16 KB activation tile
constexpr int W_BYTES = 128 * BK * 2;        // 16 KB fp16 weight tile (this CTA's 128 features)
constexpr int STAGE = X_BYTES + W_BYTES;
constexpr int SLOT = 32 * 128;               // 32 rows x 128 B, 128-byte swizzled
constexpr int SIG = 16;                      // bytes of one relayed signal

struct Smem {
    uint64_t* bars;
    uint32_t* tmem_slot;
    int* abort;
    int* g_tile;
    int* g_row;
    int* g_cnt;
    uint8_t* stages;
    uint8_t* raw;
    uint8_t* staging;
    uint8_t* sig;  // [0, PS): FULL sinks, [PS, PS+2): ACC_EMPTY sinks, PS+2: source
};

// Shared-memory plan and barrier indices for PS A+B stages and PR raw weight stages
// (PR = 0: fp16 weights loaded by TMA, no raw stage).
template <int PS_, int PR_, int NSLOT_, int KS_ = 1>
struct Lay {
    static constexpr int PS = PS_, PR = PR_;
    static constexpr int KS = KS_;                              // 64-wide K atoms per A+B stage
    static constexpr int STAGE_T = KS * STAGE;
    static constexpr int NSLOT = NSLOT_;                        // staging slots per epilogue warp
    static constexpr int STAGING = 4 * EPI_WG * NSLOT * SLOT;
    static constexpr int NB = 2 * PS + 4 + 1 + 2 * PR + PS + 2;
    static constexpr int SIG_BYTES = (PS + 2 + 1) * SIG;  // sinks for FULL[s], ACC_EMPTY[b] + one source
    static constexpr size_t SMEM = 1024 + (size_t)PS * STAGE_T + (size_t)PR * RAW_STAGE + STAGING + SIG_BYTES +
                                   NB * 8 + 16 + 3 * (MAXG + 1) * 4;
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
    static_assert(PR % DEQ_WG == 0, "raw stages must map to one dequant warpgroup each");
    static_assert((PS * STAGE_T + PR * RAW_STAGE) % 1024 == 0, "staging slots must stay 1024-byte aligned");
    static_assert(KS == 1 || PR == 0, "several K atoms per stage only with fp16 planes");

    static CEB_DEV int B_FULL(int s) { return s; }
    static CEB_DEV int B_EMPTY(int s) { return PS + s; }
    static CEB_DEV int B_ACC_FULL(int b) { return 2 * PS + b; }
    static CEB_DEV int B_ACC_EMPTY(int b) { return 2 * PS + 2 + b; }
    static CEB_DEV int B_DRAIN() { return 2 * PS + 4; }
    static CEB_DEV int B_RAW_FULL(int r) { return 2 * PS + 5 + r; }
    static CEB_DEV int B_RAW_EMPTY(int r) { return 2 * PS + 5 + PR + r; }
    static CEB_DEV int B_W_FULL(int s) { return 2 * PS + 5 + 2 * PR + s; }    // rank 1 only
    static CEB_DEV int B_ACC_FREE(int b) { return 3 * PS + 5 + 2 * PR + b; }  // rank 1 only

    static CEB_DEV Smem carve(uint8_t* base) {
        Smem s;
        uintptr_t p = (reinterpret_cast<uintptr_t>(base) + 1023) & ~uintptr_t(1023);
        s.stages = reinterpret_cast<uint8_t*>(p);
        p += (size_t)PS * STAGE_T;
        s.raw = reinterpret_cast<uint8_t*>(p);
        p += (size_t)PR * RAW_STAGE;
        s.staging = reinterpret_cast<uint8_t*>(p);
        p += STAGING;
        s.sig = reinterpret_cast<uint8_t*>(p);
        p += SIG_BYTES;
        s.bars = reinterpret_cast<uint64_t*>(p);
        p += NB * 8;
        s.tmem_slot = reinterpret_cast<uint32_t*>(p);
        s.abort = reinterpret_cast<int*>(p + 4);
        p += 16;
        s.g_tile = reinterpret_cast<int*>(p);
        s.g_row = s.g_tile + (MAXG + 1);
        s.g_cnt = s.g_row + (MAXG + 1);
        return s;
    }
};
// fp16 planes: stages of two 64-wide K atoms (64 KB: one barrier round trip per 128 K),
// three of them, one staging slot per epilogue warp.  Measured at M = 70,825 against five
// one-atom stages with two slots: qkv 1151 -> 1232, attention-out 1046 -> 1108, fc1 + GELU
// 1044 -> 1057, fc2 1242 -> 1314 TFLOP/s; two two-atom stages with two slots lose on all
// but fc1.
#ifndef CEB_PAIR_PS_F16
#define CEB_PAIR_PS_F16 3
#endif
#ifndef CEB_PAIR_SLOTS_F16
#define CEB_PAIR_SLOTS_F16 1
#endif
#ifndef CEB_PAIR_KS_F16
#define CEB_PAIR_KS_F16 2
#endif
// quantized weights: 4 A+B stages + 4 raw stages; fp16 weights: the raw bytes become more A+B stages
template <int FMT>
using LayOf = Lay<FMT == CEB_W_F16 ? CEB_PAIR_PS_F16 : 4, FMT == CEB_W_F16 ? 0 : 4, FMT == CEB_W_F16 ? CEB_PAIR_SLOTS_F16 : 1,
                  FMT == CEB_W_F16 ? CEB_PAIR_KS_F16 : 1>;

struct Tile {
    int g, fp, row0, rows;  // group, feature-pair tile, first token of the pair tile, tokens in it (<= 256)
};
CEB_DEV Tile decode(const Smem& S_, int G, int n_fp, int t) {
    int g = 0;
    while (g + 1 < G && t >= S_.g_tile[g + 1]) ++g;
    const int local = t - S_.g_tile[g];
    Tile ti;
    ti.g = g;
    ti.fp = local % n_fp;
    const int tt = local / n_fp;
    ti.row0 = S_.g_row[g] + tt * 2 * TOK;
    const int rem = S_.g_cnt[g] - tt * 2 * TOK;
    ti.rows = rem < 2 * TOK ? rem : 2 * TOK;
    return ti;
}

// one 32-row x 32-column fp32 accumulator block -> bias (+GELU), in place: the
// accumulator bits become the float results (no second 32-register array)
// PACKED: fp32 pairs, half the instructions of the scalar form and the same results
// (the fp16-plane kernel; the quantized-plane kernels, capped at 96 registers a thread,
// keep the scalar form, which needs fewer live registers)
template <bool PACKED>
CEB_DEV void epi_math(uint32_t (&v)[32], const float* bias, bool gelu) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
        float4 b = bias ? __ldg(reinterpret_cast<const float4*>(bias + j)) : make_float4(0.f, 0.f, 0.f, 0.f);
        float x0, x1, x2, x3;
        if constexpr (PACKED) {
            f32x2 xa = f2_add(f2_pack(__uint_as_float(v[j]), __uint_as_float(v[j + 1])), f2_pack(b.x, b.y));
            f32x2 xb = f2_add(f2_pack(__uint_as_float(v[j + 2]), __uint_as_float(v[j + 3])), f2_pack(b.z, b.w));
            if (gelu) {
                xa = gelu_as2(xa);
                xb = gelu_as2(xb);
            }
            f2_unpack(xa, x0, x1);
            f2_unpack(xb, x2, x3);
        } else {
            x0 = __uint_as_float(v[j]) + b.x;
            x1 = __uint_as_float(v[j + 1]) + b.y;
            x2 = __uint_as_float(v[j + 2]) + b.z;
            x3 = __uint_as_float(v[j + 3]) + b.w;
            if (gelu) {
                x0 = gelu_as(x0);
                x1 = gelu_as(x1);
                x2 = gelu_as(x2);
                x3 = gelu_as(x3);
            }
        }
        v[j] = __float_as_uint(x0);
        v[j + 1] = __float_as_uint(x1);
        v[j + 2] = __float_as_uint(x2);
        v[j + 3] = __float_as_uint(x3);
    }
}

}  // namespace pair

// Warps of the pair kernel: 4 control warps, the dequant warpgroups (quantized planes
// only) and the epilogue warpgroups.  With fp16 planes the block has no dequant warps
// (384 threads), so each thread may hold up to 168 registers instead of 102: fc1 + GELU
// 1053 -> 1068 TFLOP/s at M = 70,825, the other shapes within 1 %.
template <int FMT>
struct PairWarps {
    static constexpr int EPI0 = FMT == CEB_W_F16 ? DEQ_WARP0 : EPI_WARP0;  // first epilogue warp (a multiple of 4)
    static constexpr int THREADS = 32 * (EPI0 + 4 * EPI_WG);
};

template <int FMT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairWarps<FMT>::THREADS, 1)
    ceb_gemm_pair_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap omap,
                         const __grid_constant__ CUtensorMap wmap, const ceb_wplane w, const ceb_gemm_args a) {
    using namespace pair;
    // fp16 weight blocks are already the MMA's swizzled image: both CTAs load them with
    // the pair TMA straight into the weight stage, counted on the leader's FULL barrier
    // (no raw stage, no dequant warps, no relayed signal).
    constexpr bool kTmaW = FMT == CEB_W_F16;
    using L = LayOf<FMT>;
    constexpr int PS = L::PS, PR = L::PR, NB = L::NB;
    extern __shared__ uint8_t smem_raw[];
    const Smem SH = L::carve(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int G = a.offsets ? w.n_groups : 1;
    const int n_fp = w.n_out / FEAT;
    const int n_ftiles = w.n_out / BM;
    const int nkb = w.k / BK;
    const int pair_id = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NB; ++i) {
            uint32_t cnt = 1;
            if (i < PS) cnt = kTmaW ? 1 : 1 + 4;                            // expect_tx (+ leader dequant warps)
            if (i >= 2 * PS + 2 && i < 2 * PS + 4) cnt = 4 * EPI_WG;        // leader epilogue warps (one with expect_tx)
            if (i >= 2 * PS + 5 + PR && i < 2 * PS + 5 + 2 * PR) cnt = 4;   // this CTA's dequant warpgroup
            if (i >= L::B_W_FULL(0) && i < L::B_W_FULL(0) + PS) cnt = 4;          // rank 1's dequant warpgroup
            if (i >= L::B_ACC_FREE(0) && i < L::B_ACC_FREE(0) + 2) cnt = 4 * EPI_WG;  // rank 1's epilogue warps
            mbar_init(smem_u32(&SH.bars[i]), cnt);
        }
        fence_mbar_init();
        *SH.abort = 0;
        *reinterpret_cast<uint4*>(SH.sig + (PS + 2) * SIG) = make_uint4(0, 0, 0, 0);  // signal source
        fence_proxy_async_smem();
        int tiles = 0;
        for (int g = 0; g < G; ++g) {
            int r0 = a.offsets ? a.offsets[g] : 0;
            int r1 = a.offsets ? a.offsets[g + 1] : a.m_rows;
            if (r0 < 0 || r1 < r0 || r1 > a.m_rows) {
                if (a.err) atomicCAS(a.err, 0, (int)CEB_DEVERR_BAD_GROUP);
                r0 = r1 = 0;
            }
            SH.g_tile[g] = tiles;
            SH.g_row[g] = r0;
            SH.g_cnt[g] = r1 - r0;
            tiles += ((r1 - r0 + 2 * TOK - 1) / (2 * TOK)) * n_fp;
        }
        SH.g_tile[G] = tiles;
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&xmap);
        tma_prefetch_desc(&omap);
        if (kTmaW) tma_prefetch_desc(&wmap);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(SH.tmem_slot), TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // barriers of both CTAs initialised before any remote arrive
    tc_fence_after();
    const uint32_t tmem = *SH.tmem_slot;
    const int total = SH.g_tile[G];
    volatile int* abort = SH.abort;
    auto bar = [&](int i) { return smem_u32(&SH.bars[i]); };
    auto lead_bar = [&](int i) { return mapa_shared(bar(i), 0); };
    auto wait_at = [&](int i, uint32_t parity, int code) {
        return mbar_wait(bar(i), parity, abort, a.err, code | ((i + 1) << 16));
    };
    auto wait_cl = [&](int i, uint32_t parity, int code) {
        return mbar_wait_cluster(bar(i), parity, abort, a.err, code | ((i + 1) << 16));
    };
    constexpr int KS = L::KS;  // 64-wide K atoms per stage: stage s holds KS activation atoms, then KS weight atoms
    const int nst = nkb / KS;  // stages per tile
    auto x_stage = [&](int s) { return SH.stages + (size_t)s * L::STAGE_T; };
    auto w_stage = [&](int s) { return SH.stages + (size_t)s * L::STAGE_T + KS * X_BYTES; };
    auto wblock = [&](const Tile& ti, int kb) {
        const int ft = 2 * ti.fp + (int)rank;  // this CTA's 128-feature weight tile
        return w.q + (((size_t)ti.g * n_ftiles + ft) * nkb + kb) * (size_t)w.blk_bytes;
    };

    if (warp == 0) {
        // ------------------------------------------------ activation tiles (this CTA's 128 tokens)
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int t = pair_id; t < total && ok; t += n_pairs) {
                const Tile ti = pair::decode(SH, G, n_fp, t);
                for (int ks = 0; ks < nst; ++ks, ++it) {
                    const int s = it % PS;
                    if (!wait_at(L::B_EMPTY(s), ((it / PS) & 1) ^ 1, CEB_DEVERR_TIMEOUT_TMA)) {
                        ok = false;
                        break;
                    }
                    if (leader)
                        mbar_arrive_expect_tx(bar(L::B_FULL(s)), kTmaW ? 2 * KS * (X_BYTES + W_BYTES) : 2 * X_BYTES + SIG);
#pragma unroll
                    for (int a = 0; a < KS; ++a)
                        tma_load_2d_pair(smem_u32(x_stage(s) + a * X_BYTES), &xmap, lead_bar(L::B_FULL(s)),
                                         (ks * KS + a) * BK, ti.row0 + TOK * (int)rank);
                }
            }
            if (!ok && leader) {  // let issued copies land before the CTA can exit
                const uint32_t n = it < PS ? it : PS;
                for (uint32_t i = it - n; i < it; ++i)
                    mbar_wait_cluster(bar(L::B_FULL(i % PS)), (i / PS) & 1, nullptr, nullptr, 0);
            }
        }
    } else if (warp == 1 && !leader) {
        // ------------------------------------------------ relay: rank 1's weight tiles ready -> leader's FULL
        if (lane == 0 && !kTmaW) {
            const int my_tiles = pair_id < total ? (total - 1 - pair_id) / n_pairs + 1 : 0;
            const uint32_t n_items = (uint32_t)(my_tiles * nkb);
            for (uint32_t it = 0; it < n_items; ++it) {
                const int s = it % PS;
                if (!wait_at(L::B_W_FULL(s), (it / PS) & 1, CEB_DEVERR_TIMEOUT_DEQ)) break;
                bulk_copy_to_cluster(mapa_shared(smem_u32(SH.sig + s * SIG), 0), smem_u32(SH.sig + (PS + 2) * SIG),
                                     SIG, lead_bar(L::B_FULL(s)));
            }
        }
    } else if (warp == 3 && !leader) {
        // ------------------------------------------------ relay: rank 1's accumulator drained -> leader's ACC_EMPTY
        if (lane == 0) {
            uint32_t lt = 0;
            for (int t = pair_id; t < total; t += n_pairs, ++lt) {
                const int ab = lt & 1;
                if (!wait_at(L::B_ACC_FREE(ab), (lt >> 1) & 1, CEB_DEVERR_TIMEOUT_EPI)) break;
                bulk_copy_to_cluster(mapa_shared(smem_u32(SH.sig + (PS + ab) * SIG), 0),
                                     smem_u32(SH.sig + (PS + 2) * SIG), SIG, lead_bar(L::B_ACC_EMPTY(ab)));
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer (leader only)
        if (lane == 0) {
            const uint32_t idesc = idesc_f16_f32(2 * TOK, FEAT);
            uint32_t it = 0, lt = 0;
            bool ok = true;
            for (int t = pair_id; t < total && ok; t += n_pairs, ++lt) {
                const int ab = lt & 1;
                if (!wait_cl(L::B_ACC_EMPTY(ab), ((lt >> 1) & 1) ^ 1, CEB_DEVERR_TIMEOUT_MMA)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + (uint32_t)(ab * FEAT);
                for (int ks = 0; ks < nst; ++ks, ++it) {
                    const int s = it % PS;
                    if (!wait_cl(L::B_FULL(s), (it / PS) & 1, CEB_DEVERR_TIMEOUT_MMA)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int a = 0; a < KS; ++a) {
                        const uint64_t adesc = smem_desc_sw128(smem_u32(x_stage(s) + a * X_BYTES));
                        const uint64_t bdesc = smem_desc_sw128(smem_u32(w_stage(s) + a * W_BYTES));
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk)
                            mma_pair_f16_ss(d_tmem, adesc + (uint64_t)(kk * 2), bdesc + (uint64_t)(kk * 2), idesc,
                                            (ks | a | kk) != 0);
                    }
                    mma_pair_commit(bar(L::B_EMPTY(s)));
                    mma_pair_commit(mapa_shared(bar(L::B_EMPTY(s)), 1));
                }
                if (ok) {
                    mma_pair_commit(bar(L::B_ACC_FULL(ab)));
                    mma_pair_commit(mapa_shared(bar(L::B_ACC_FULL(ab)), 1));
                }
            }
            // rank 1's last ACC_EMPTY signals (16-byte copies into this CTA) have landed
            for (uint32_t l = lt >= 2 ? lt - 2 : 0; l < lt; ++l)
                mbar_wait_cluster(bar(L::B_ACC_EMPTY(l & 1)), (l >> 1) & 1, nullptr, nullptr, 0);
            // every issued MMA (they write both CTAs' tensor memory) retires before TMEM is released
            mma_pair_commit(bar(L::B_DRAIN()));
            mbar_wait(bar(L::B_DRAIN()), 0, nullptr, nullptr, 0);
        }
    } else if (warp == 2 && kTmaW) {
        // ------------------------------------------------ weight loader (fp16 blocks, pair TMA)
        if (lane == 0) {
            uint32_t it = 0;
            for (int t = pair_id; t < total; t += n_pairs) {
                const Tile ti = pair::decode(SH, G, n_fp, t);
                const int ft = 2 * ti.fp + (int)rank;
                bool ok = true;
                for (int ks = 0; ks < nst; ++ks, ++it) {
                    const int s = it % PS;
                    if (!wait_at(L::B_EMPTY(s), ((it / PS) & 1) ^ 1, CEB_DEVERR_TIMEOUT_TMA)) {
                        ok = false;
                        break;
                    }
                    // block (g, ft, kb) is rows [128 * index, +128) of the [blocks * 128, 64] fp16 view
#pragma unroll
                    for (int a = 0; a < KS; ++a)
                        tma_load_2d_pair(smem_u32(w_stage(s) + a * W_BYTES), &wmap, lead_bar(L::B_FULL(s)), 0,
                                         (int)((((size_t)ti.g * n_ftiles + ft) * nkb + ks * KS + a) * 128));
                }
                if (!ok) break;
            }
        }
    } else if (warp == 2) {
        // ------------------------------------------------ weight loader (this CTA's quantized blocks)
        if constexpr (!kTmaW) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int t = pair_id; t < total && ok; t += n_pairs) {
                const Tile ti = pair::decode(SH, G, n_fp, t);
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int rs = it % PR;
                    if (!wait_at(L::B_RAW_EMPTY(rs), ((it / PR) & 1) ^ 1, CEB_DEVERR_TIMEOUT_TMA)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(bar(L::B_RAW_FULL(rs)), (uint32_t)w.blk_bytes);
                    bulk_load(smem_u32(SH.raw + (size_t)rs * RAW_STAGE), wblock(ti, kb), (uint32_t)w.blk_bytes,
                              bar(L::B_RAW_FULL(rs)));
                }
            }
            if (!ok) {
                const uint32_t n = it < PR ? it : PR;
                for (uint32_t i = it - n; i < it; ++i)
                    mbar_wait(bar(L::B_RAW_FULL(i % PR)), (i / PR) & 1, nullptr, nullptr, 0);
            }
        }
        }
    } else if (!kTmaW && warp >= DEQ_WARP0 && warp < EPI_WARP0) {
        // ------------------------------------------------ dequant (raw stage -> fp16 weight stage)
        if constexpr (!kTmaW) {
        const int wg = (warp - DEQ_WARP0) >> 2;
        const int r = 32 * (warp & 3) + lane;
        const int my_tiles = pair_id < total ? (total - 1 - pair_id) / n_pairs + 1 : 0;
        const int n_items = my_tiles * nkb;
        for (int i = wg; i < n_items; i += DEQ_WG) {
            const int rs = i % PR, s = i % PS;
            if (!__all_sync(0xffffffffu, wait_at(L::B_RAW_FULL(rs), (i / PR) & 1, CEB_DEVERR_TIMEOUT_DEQ))) break;
            Raw<FMT> raw;
            load_raw_smem<FMT>(SH.raw + (size_t)rs * RAW_STAGE, r, raw);
            uint32_t o[32];
            convert<FMT>(raw, o);
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(L::B_RAW_EMPTY(rs)));
            if (!__all_sync(0xffffffffu, wait_at(L::B_EMPTY(s), ((i / PS) & 1) ^ 1, CEB_DEVERR_TIMEOUT_DEQ))) break;
            uint8_t* row = w_stage(s) + r * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) =
                    make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(leader ? L::B_FULL(s) : L::B_W_FULL(s)));
        }
        }
    } else if (warp >= PairWarps<FMT>::EPI0) {
        // ------------------------------------------------ epilogue (this CTA's 128 tokens)
        const int ew = warp - PairWarps<FMT>::EPI0;
        const int wg = ew >> 2;                 // columns (features) 128*wg .. 128*wg+127 of the pair tile
        const int q = warp & 3;                 // TMEM lanes (tokens) 32q .. 32q+31
        const uint32_t lane_addr = (uint32_t)(32 * q) << 16;
        const bool f16 = (a.epi & CEB_EPI_F16_OUT) != 0, gelu = (a.epi & CEB_EPI_GELU) != 0;
        constexpr int NSLOT = L::NSLOT;
        uint32_t lt = 0, nstore = 0;
        for (int t = pair_id; t < total; t += n_pairs, ++lt) {
            const Tile ti = pair::decode(SH, G, n_fp, t);
            const int ab = lt & 1;
            if (!__all_sync(0xffffffffu, wait_at(L::B_ACC_FULL(ab), (lt >> 1) & 1, CEB_DEVERR_TIMEOUT_EPI))) break;
            tc_fence_after();
            const int my_rows = ti.rows - TOK * (int)rank;   // tokens of the pair tile held by this CTA
            const int lim = my_rows - 32 * q;                 // valid rows of this warp's 32
            const int row = ti.row0 + TOK * (int)rank + 32 * q;
            const int f_base = ti.fp * FEAT + 128 * wg;
            const float* bias = (a.epi & CEB_EPI_BIAS) ? a.bias + (size_t)ti.g * a.bias_group_stride : nullptr;
            const uint32_t col0 = (uint32_t)(ab * FEAT + 128 * wg);
            const int chunk_cols = f16 ? 64 : 32;
            for (int c0 = 0; c0 < 128; c0 += chunk_cols) {
                if (lim <= 0) break;
                const bool full = lim >= 32;
                // slots are used in turn; the store that last used this one has finished reading it
                uint8_t* slot = SH.staging + (size_t)(ew * NSLOT + (int)(nstore % NSLOT)) * SLOT;
                const uint32_t slot_u32 = smem_u32(slot);
                if (kTmaW && gelu && f16) {
                    // fc1 + GELU: the chunk's TMEM loads and GELU run before the wait for the store
                    // that last used this slot, so that store's read of shared memory hides behind
                    // the math (+4.5 % at M = 70,825). Without GELU the math is short and the
                    // branch below, which writes each 32-column half as soon as it is ready,
                    // measured ~1 % faster.
                    uint32_t p[32];  // the chunk's 64 columns as 32 packed fp16 pairs
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        uint32_t v[32];
                        tmem_ld32(tmem + lane_addr + col0 + (uint32_t)(c0 + 32 * h), v);
                        tmem_ld_wait();
                        epi_math<true>(v, bias ? bias + f_base + c0 + 32 * h : nullptr, true);
                        const float* x = reinterpret_cast<const float*>(v);
#pragma unroll
                        for (int j = 0; j < 16; ++j) p[16 * h + j] = h2_as_u32(__floats2half2_rn(x[2 * j], x[2 * j + 1]));
                    }
                    if (full) {
                        if (nstore >= NSLOT) {
                            if (lane == 0) bulk_wait_read<NSLOT - 1>();
                            __syncwarp();
                        }
#pragma unroll
                        for (int c = 0; c < 8; ++c)
                            *reinterpret_cast<uint4*>(slot + lane * 128 + ((c ^ (lane & 7)) << 4)) =
                                make_uint4(p[4 * c], p[4 * c + 1], p[4 * c + 2], p[4 * c + 3]);
                    } else if (lane < lim) {
                        uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(a.out) +
                                                            (size_t)(row + lane) * a.ldo + f_base + c0);
#pragma unroll
                        for (int c = 0; c < 8; ++c) o[c] = make_uint4(p[4 * c], p[4 * c + 1], p[4 * c + 2], p[4 * c + 3]);
                    }
                } else {
                    if (full && nstore >= NSLOT) {
                        if (lane == 0) bulk_wait_read<NSLOT - 1>();
                        __syncwarp();
                    }
                    for (int h = 0; h < chunk_cols; h += 32) {
                        uint32_t v[32];
                        tmem_ld32(tmem + lane_addr + col0 + (uint32_t)(c0 + h), v);
                        tmem_ld_wait();
                        epi_math<kTmaW>(v, bias ? bias + f_base + c0 + h : nullptr, gelu);
                        const float* x = reinterpret_cast<const float*>(v);
                        if (f16) {
                            uint32_t p[16];
    #pragma unroll
                            for (int j = 0; j < 16; ++j) p[j] = h2_as_u32(__floats2half2_rn(x[2 * j], x[2 * j + 1]));
                            if (full) {  // 64 B = chunks 4*(h/32) .. +3 of the 128-B swizzled row
    #pragma unroll
                                for (int c = 0; c < 4; ++c) {
                                    const int cc = c + (h >> 3);
                                    *reinterpret_cast<uint4*>(slot + lane * 128 + ((cc ^ (lane & 7)) << 4)) =
                                        make_uint4(p[4 * c], p[4 * c + 1], p[4 * c + 2], p[4 * c + 3]);
                                }
                            } else if (lane < lim) {
                                uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(a.out) +
                                                                    (size_t)(row + lane) * a.ldo + f_base + c0 + h);
    #pragma unroll
                                for (int c = 0; c < 4; ++c) o[c] = make_uint4(p[4 * c], p[4 * c + 1], p[4 * c + 2], p[4 * c + 3]);
                            }
                        } else {
                            if (full) {
    #pragma unroll
                                for (int c = 0; c < 8; ++c)
                                    *reinterpret_cast<float4*>(slot + lane * 128 + ((c ^ (lane & 7)) << 4)) =
                                        make_float4(x[4 * c], x[4 * c + 1], x[4 * c + 2], x[4 * c + 3]);
                            } else if (lane < lim) {
                                float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(a.out) +
                                                                      (size_t)(row + lane) * a.ldo + f_base + c0 + h);
    #pragma unroll
                                for (int c = 0; c < 8; ++c) o[c] = make_float4(x[4 * c], x[4 * c + 1], x[4 * c + 2], x[4 * c + 3]);
                            }
                        }
                    }
                }
                if (full) {
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&omap, slot_u32, f_base + c0, row);
                        bulk_commit();
                    }
                    ++nstore;
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (!leader)
                    mbar_arrive(bar(L::B_ACC_FREE(ab)));
                else if (ew == 0)
                    mbar_arrive_expect_tx(bar(L::B_ACC_EMPTY(ab)), SIG);  // + rank 1's relayed signal
                else
                    mbar_arrive(bar(L::B_ACC_EMPTY(ab)));
            }
        }
        if (lane == 0) bulk_wait<0>();  // output stores complete before the CTA retires
    }

    tc_fence_before();
    __syncwarp();
    cluster_sync();  // no remote arrive or MMA can still target this CTA once it passes here
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, TMEM_COLS);
    }
}

template <int FMT>
int launch_pair(const CUtensorMap& xmap, const CUtensorMap& omap, const CUtensorMap& wmap, const ceb_wplane& w,
                const ceb_gemm_args& a, int max_pairs, cudaStream_t st) {
    static int resident_of[CEB_MAX_DEVICES] = {};  // co-resident pairs, per device
    int& pairs_resident = resident_of[ceb_device_index()];
    if (!pairs_resident) {
        if (int rc = ceb_func_smem(reinterpret_cast<const void*>(ceb_gemm_pair_kernel<FMT>), pair::LayOf<FMT>::SMEM))
            return rc;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * ceb_num_sms(), 1, 1);
        cfg.blockDim = dim3(PairWarps<FMT>::THREADS, 1, 1);
        cfg.dynamicSmemBytes = pair::LayOf<FMT>::SMEM;
        int n = 0;  // cluster size comes from the kernel's __cluster_dims__
        CEB_CUDA_OK(cudaOccupancyMaxActiveClusters(&n, ceb_gemm_pair_kernel<FMT>, &cfg));
        pairs_resident = n > 0 ? n : 1;
    }
    int pairs = pairs_resident < max_pairs ? pairs_resident : max_pairs;
    if (pairs < 1) pairs = 1;
    ceb_gemm_pair_kernel<FMT><<<2 * pairs, PairWarps<FMT>::THREADS, pair::LayOf<FMT>::SMEM, st>>>(xmap, omap, wmap, w,
                                                                                                a);
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}


// One CTA per block, thread = row: a quantized block -> the fp16 block of the same
// (group, feature tile, k-block), through the GEMM's own dequantizer, so the values
// are the fp16 numbers the dequant warps would have put in shared memory.
template <int FMT>
__global__ void expand_f16_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t src_blk) {
    const int r = threadIdx.x;
    const uint8_t* blk = src + (size_t)blockIdx.x * src_blk;
    Raw<FMT> raw;
    load_raw_smem<FMT>(blk, r, raw);  // generic pointer: the block layout is the same in global memory
    uint32_t o[32];
    convert<FMT>(raw, o);
    uint8_t* row = dst + (size_t)blockIdx.x * 16384 + r * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) = make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
}

}  // namespace

int ceb_wplane_expand_f16(ceb_wplane* w, cudaStream_t st) {
    if (w->format == CEB_W_F16) return 0;
    if (w->format != CEB_W_Q8_0 && w->format != CEB_W_Q4_K) return ceb_set_error(2, "expand: format %d", w->format);
    const int64_t blocks = (int64_t)w->n_groups * (w->n_out / BM) * (w->k / BK);
    if (blocks <= 0) return 0;
    if (blocks > 0x7fffffff) return ceb_set_error(2, "expand: %lld blocks", (long long)blocks);
    ceb_wplane e = *w;
    e.format = CEB_W_F16;
    e.blk_bytes = ceb_wblock_bytes(CEB_W_F16);
    e.q_bytes = (size_t)blocks * (size_t)e.blk_bytes;
    e.s_bytes = 0;
    if (cudaMalloc(&e.q, e.q_bytes) != cudaSuccess) {
        cudaGetLastError();
        return ceb_set_error(4, "expand: out of device memory (%zu bytes)", e.q_bytes);
    }
    if (w->format == CEB_W_Q8_0)
        expand_f16_kernel<CEB_W_Q8_0><<<(unsigned)blocks, BM, 0, st>>>(w->q, e.q, w->blk_bytes);
    else
        expand_f16_kernel<CEB_W_Q4_K><<<(unsigned)blocks, BM, 0, st>>>(w->q, e.q, w->blk_bytes);
    cudaError_t err = cudaGetLastError();
    if (err == cudaSuccess) err = cudaStreamSynchronize(st);
    if (err != cudaSuccess) {
        cudaFree(e.q);
        return ceb_set_cuda_error(err, "expand", __FILE__, __LINE__);
    }
    ceb_wplane_free(w);
    *w = e;
    return 0;
}

// The CTA-pair kernel takes weights whose output width is a multiple of 256 (every
// linear layer of the supported encoders) in any plane format; narrower or odd
// widths and unaligned bias vectors use the single-CTA kernel.  Setting
// CEB_GEMM_SINGLE_CTA=1 in the environment forces the single-CTA kernel.
static bool ceb_gemm_use_pairs(const ceb_wplane& w, const ceb_gemm_args& a) {
    static const bool forced_single = [] {
        const char* e = getenv("CEB_GEMM_SINGLE_CTA");
        return e && e[0] == '1';
    }();
    if (forced_single) return false;
    if (w.n_out % pair::FEAT) return false;
    if (w.format == CEB_W_F16 && (w.k / BK) % CEB_PAIR_KS_F16) return false;  // whole stages of K atoms
    if ((a.epi & CEB_EPI_BIAS) &&
        ((reinterpret_cast<uintptr_t>(a.bias) & 15) || (a.offsets && (a.bias_group_stride & 3))))
        return false;
    return true;
}

int ceb_gemm_launch(const ceb_wplane& w, const void* act_f16, int act_rows, const ceb_gemm_args& a,
                    cudaStream_t stream, int max_ctas) {
    if (w.n_out % BM || w.k % BK || w.k <= 0 || w.n_out <= 0)
        return ceb_set_error(2, "gemm: n_out=%d must be a multiple of %d and k=%d of %d", w.n_out, BM, w.k, BK);
    if (a.offsets && (w.n_groups < 1 || w.n_groups > MAXG))
        return ceb_set_error(2, "gemm: %d groups (max %d)", w.n_groups, MAXG);
    if ((reinterpret_cast<uintptr_t>(act_f16) & 15) != 0) return ceb_set_error(2, "gemm: activations not 16-B aligned");
    if ((a.epi & CEB_EPI_F16_OUT) && (a.ldo & 1)) return ceb_set_error(2, "gemm: fp16 output stride must be even");
    if (act_rows <= 0) return 0;
    const int esz = (a.epi & CEB_EPI_F16_OUT) ? 2 : 4;
    if ((reinterpret_cast<uintptr_t>(a.out) & 15) || ((size_t)a.ldo * esz) % 16 || a.ldo < w.n_out)
        return ceb_set_error(2, "gemm: output must be 16-B aligned with a row stride >= n_out and a multiple of 16 B");
    const int groups = a.offsets ? w.n_groups : 1;
    const double flops = 2.0 * (double)a.m_rows * w.n_out * w.k;
    const double bytes = (double)(w.q_bytes + w.s_bytes) + (double)a.m_rows * w.k * 2 +
                         (double)a.m_rows * w.n_out * ((a.epi & CEB_EPI_F16_OUT) ? 2 : 4);
    CUtensorMap map, omap;
    int mrc = 0;
    if (ceb_gemm_use_pairs(w, a)) {
        // CTA-pair kernel: 128-token activation boxes, 128-byte-swizzled 32-row output boxes
        mrc = ceb_make_tmap_2d_f16(&map, act_f16, (uint64_t)w.k, (uint64_t)act_rows, (uint64_t)w.k * 2, BK, pair::TOK);
        if (mrc) return mrc;
        mrc = ceb_make_tmap_2d(&omap, a.out, esz, (uint64_t)w.n_out, (uint64_t)a.m_rows, (uint64_t)a.ldo * esz,
                               esz == 2 ? 64 : 32, 32, true);
        if (mrc) return mrc;
        const int n_fp = w.n_out / pair::FEAT;
        long long bound = (long long)n_fp * ((act_rows + 2 * pair::TOK - 1) / (2 * pair::TOK) + groups);
        int max_pairs = ceb_num_sms() / 2;
        if (max_ctas > 0 && max_ctas / 2 < max_pairs) max_pairs = max_ctas / 2 > 0 ? max_ctas / 2 : 1;
        if (bound < max_pairs) max_pairs = (int)bound;
        CUtensorMap wmap = {};
        if (w.format == CEB_W_F16) {  // the plane as [blocks * 128 rows, 64] fp16, blocks already swizzled
            const uint64_t blocks = (uint64_t)w.n_groups * (w.n_out / BM) * (w.k / BK);
            mrc = ceb_make_tmap_2d(&wmap, w.q, 2, (uint64_t)BK, blocks * BM, (uint64_t)BK * 2, BK, BM, false);
            if (mrc) return mrc;
        }
        int rc = 0;
        switch (w.format) {
            case CEB_W_Q8_0: CEB_LAUNCH(a.prof_cat, stream, flops, bytes, rc = launch_pair<CEB_W_Q8_0>(map, omap, wmap, w, a, max_pairs, stream)); break;
            case CEB_W_Q4_K: CEB_LAUNCH(a.prof_cat, stream, flops, bytes, rc = launch_pair<CEB_W_Q4_K>(map, omap, wmap, w, a, max_pairs, stream)); break;
            case CEB_W_F16: CEB_LAUNCH(a.prof_cat, stream, flops, bytes, rc = launch_pair<CEB_W_F16>(map, omap, wmap, w, a, max_pairs, stream)); break;
            default: return ceb_set_error(2, "gemm: unknown weight format %d", w.format);
        }
        return rc;
    }
    mrc = ceb_make_tmap_2d_f16(&map, act_f16, (uint64_t)w.k, (uint64_t)act_rows, (uint64_t)w.k * 2, BK, BN);
    if (mrc) return mrc;
    mrc = ceb_make_tmap_2d(&omap, a.out, esz, (uint64_t)w.n_out, (uint64_t)a.m_rows, (uint64_t)a.ldo * esz, 32, 32,
                           false);
    if (mrc) return mrc;
    const int n_ftiles = w.n_out / BM;
    long long bound = (long long)n_ftiles * ((act_rows + BN - 1) / BN + groups);
    int grid = ceb_num_sms();
    if (max_ctas > 0 && max_ctas < grid) grid = max_ctas;
    if (bound < grid) grid = (int)bound;
    int rc = 0;
    switch (w.format) {
        case CEB_W_Q8_0: CEB_LAUNCH(a.prof_cat, stream, flops, bytes, rc = launch_fmt<CEB_W_Q8_0>(map, omap, w, a, grid, stream)); break;
        case CEB_W_Q4_K: CEB_LAUNCH(a.prof_cat, stream, flops, bytes, rc = launch_fmt<CEB_W_Q4_K>(map, omap, w, a, grid, stream)); break;
        case CEB_W_F16: CEB_LAUNCH(a.prof_cat, stream, flops, bytes, rc = launch_fmt<CEB_W_F16>(map, omap, w, a, grid, stream)); break;
        default: return ceb_set_error(2, "gemm: unknown weight format %d", w.format);
    }
    return rc;
}
