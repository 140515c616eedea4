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
#include <cstdio>

#include "ceb_internal.h"
#include "common.cuh"

namespace {

constexpr int BM = 128;
constexpr int BN = 256;               // activation rows (tokens) per tile = max MMA N
constexpr int BK = 64;
constexpr int S = 3;                  // pipeline stages (A + B tiles)
constexpr int R = 4;                  // raw (still quantized) weight stages
constexpr int RAW_STAGE = 8704;       // largest quantized block (Q8_0)
constexpr int MAXG = 64;
constexpr int A_STAGE_BYTES = BM * BK * 2;   // 16 KB, written by the dequant warps
constexpr int B_STAGE_BYTES = BN * BK * 2;   // 32 KB, written by TMA
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr uint32_t TMEM_COLS = 512;          // two BN-column fp32 accumulators
constexpr int DEQ_WG = 2, EPI_WG = 2;
constexpr int DEQ_WARP0 = 4, EPI_WARP0 = DEQ_WARP0 + 4 * DEQ_WG;
constexpr int NTHREADS = 32 * (EPI_WARP0 + 4 * EPI_WG);
constexpr int STAGING_SLOT = 32 * 32 * 4;    // one 32x32 fp32 output block per slot
constexpr int STAGING_BYTES = 4 * EPI_WG * STAGING_SLOT;  // one slot per epilogue warp
static_assert(2 * BN <= (int)TMEM_COLS, "TMEM budget");

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
                if (lim >= 32) {
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
    static bool attr_set = false;
    if (!attr_set) {
        CEB_CUDA_OK(cudaFuncSetAttribute(ceb_gemm_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)SMEM_BYTES));
        attr_set = true;
    }
    ceb_gemm_kernel<FMT><<<grid, NTHREADS, SMEM_BYTES, st>>>(map, omap, w, a);
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

}  // namespace

int ceb_gemm_launch(const ceb_wplane& w, const void* act_f16, int act_rows, const ceb_gemm_args& a,
                    cudaStream_t stream, int max_ctas) {
    if (w.n_out % BM || w.k % BK || w.k <= 0 || w.n_out <= 0)
        return ceb_set_error(2, "gemm: n_out=%d must be a multiple of %d and k=%d of %d", w.n_out, BM, w.k, BK);
    if (a.offsets && (w.n_groups < 1 || w.n_groups > MAXG))
        return ceb_set_error(2, "gemm: %d groups (max %d)", w.n_groups, MAXG);
    if ((reinterpret_cast<uintptr_t>(act_f16) & 15) != 0) return ceb_set_error(2, "gemm: activations not 16-B aligned");
    if ((a.epi & CEB_EPI_F16_OUT) && (a.ldo & 1)) return ceb_set_error(2, "gemm: fp16 output stride must be even");
    if (act_rows <= 0) return 0;
    CUtensorMap map, omap;
    int mrc = ceb_make_tmap_2d_f16(&map, act_f16, (uint64_t)w.k, (uint64_t)act_rows, (uint64_t)w.k * 2, BK, BN);
    if (mrc) return mrc;
    const int esz = (a.epi & CEB_EPI_F16_OUT) ? 2 : 4;
    if ((reinterpret_cast<uintptr_t>(a.out) & 15) || ((size_t)a.ldo * esz) % 16 || a.ldo < w.n_out)
        return ceb_set_error(2, "gemm: output must be 16-B aligned with a row stride >= n_out and a multiple of 16 B");
    mrc = ceb_make_tmap_2d(&omap, a.out, esz, (uint64_t)w.n_out, (uint64_t)a.m_rows, (uint64_t)a.ldo * esz, 32, 32,
                           false);
    if (mrc) return mrc;
    const int n_ftiles = w.n_out / BM;
    const int groups = a.offsets ? w.n_groups : 1;
    long long bound = (long long)n_ftiles * ((act_rows + BN - 1) / BN + groups);
    int grid = ceb_num_sms();
    if (max_ctas > 0 && max_ctas < grid) grid = max_ctas;
    if (bound < grid) grid = (int)bound;
    const double flops = 2.0 * (double)a.m_rows * w.n_out * w.k;
    const double bytes = (double)(w.q_bytes + w.s_bytes) + (double)a.m_rows * w.k * 2 +
                         (double)a.m_rows * w.n_out * ((a.epi & CEB_EPI_F16_OUT) ? 2 : 4);
    int rc = 0;
    switch (w.format) {
        case CEB_W_Q8_0: CEB_LAUNCH(CEB_PROF_GEMM, stream, flops, bytes, rc = launch_fmt<CEB_W_Q8_0>(map, omap, w, a, grid, stream)); break;
        case CEB_W_Q4_K: CEB_LAUNCH(CEB_PROF_GEMM, stream, flops, bytes, rc = launch_fmt<CEB_W_Q4_K>(map, omap, w, a, grid, stream)); break;
        case CEB_W_F16: CEB_LAUNCH(CEB_PROF_GEMM, stream, flops, bytes, rc = launch_fmt<CEB_W_F16>(map, omap, w, a, grid, stream)); break;
        default: return ceb_set_error(2, "gemm: unknown weight format %d", w.format);
    }
    return rc;
}
