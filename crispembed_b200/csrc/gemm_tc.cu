// gemm_tc.cu -- grouped GEMM over block-quantized weights on tcgen05 / TMEM.
//
// Replaces the ggml_mul_mat / ggml_mul_mat_id products of the encoder graph
// (src/crispembed.cpp:1160-1177, :1320, :1333-1371, :1411-1416 of the
// reference), computing for every group g (expert, or one group for a dense
// layer) and every activation row r in the group's row range:
//
//     out[r, n] = epilogue( sum_k W_g[n, k] * X[r, k] )
//
// Operand roles ("TS" form of tcgen05.mma, A from tensor memory):
//   A = weight tile, 128 output features x 64 k, dequantized by eight warps
//       straight from global memory (Q8_0 / Q4_K / fp16 planes) into TMEM,
//       so the weights never pass through shared memory;
//   B = activation tile, up to BN rows x 64 k fp16, loaded by TMA into
//       128-byte-swizzled shared memory;
//   D = fp32 accumulator in TMEM, [128 features (lanes)] x [BN rows (columns)],
//       double buffered so the epilogue of one tile overlaps the next tile.
// TMEM budget (512 columns): 2 x BN accumulator columns + SA x 32 A-stage columns.
//
// Warp roles (640 threads, one persistent CTA per SM):
//   warp 0        TMA producer of activation stages
//   warp 1        TMEM owner + single-thread MMA issuer
//   warps 4..11   dequant producers, two warpgroups taking alternate K-blocks
//                 (thread i of a warpgroup <-> weight row / TMEM lane i)
//   warps 12..19  epilogue, two warpgroups taking alternate 32-column chunks
//                 (thread i <-> output feature i): bias, GELU, store
// Tiles (group, token tile, feature tile) are distributed round-robin; the
// group table is read from device memory, so no host synchronisation is
// needed between routing and the expert GEMMs.
#include <cstdio>

#include "ceb_internal.h"
#include "common.cuh"

namespace {

constexpr int BM = 128;
constexpr int BN = 192;               // activation rows (tokens) per tile = MMA N
constexpr int BK = 64;
constexpr int SB = 6;                 // activation smem stages
constexpr int SA = (512 - 2 * BN) / 32;  // TMEM A stages (4)
constexpr int MAXG = 64;
constexpr int B_STAGE_BYTES = BN * BK * 2;
constexpr uint32_t TMEM_COLS = 512;
constexpr int A_COL0 = 2 * BN;
constexpr int DEQ_WG = 2, EPI_WG = 2;
constexpr int DEQ_WARP0 = 4, EPI_WARP0 = DEQ_WARP0 + 4 * DEQ_WG;
constexpr int NTHREADS = 32 * (EPI_WARP0 + 4 * EPI_WG);
static_assert(SA >= 2 && A_COL0 + 32 * SA <= 512, "TMEM budget");

constexpr int NBARS = 2 * SB + 2 * SA + 4 + 1;
constexpr size_t SMEM_BYTES = 1024 /*align slack*/ + (size_t)SB * B_STAGE_BYTES + NBARS * 8 + 16 + 3 * (MAXG + 1) * 4;

struct Shared {
    uint64_t* bars;
    uint32_t* tmem_slot;
    int* abort;
    int* g_tile;
    int* g_row;
    int* g_cnt;
    uint8_t* b_stages;
};

CEB_DEV Shared carve(uint8_t* raw) {
    Shared s;
    uintptr_t p = (reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023);
    s.b_stages = reinterpret_cast<uint8_t*>(p);
    p += (size_t)SB * B_STAGE_BYTES;
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
CEB_DEV int BAR_B_FULL(int s) { return s; }
CEB_DEV int BAR_B_EMPTY(int s) { return SB + s; }
CEB_DEV int BAR_A_FULL(int s) { return 2 * SB + s; }
CEB_DEV int BAR_A_EMPTY(int s) { return 2 * SB + SA + s; }
CEB_DEV int BAR_ACC_FULL(int b) { return 2 * SB + 2 * SA + b; }
CEB_DEV int BAR_ACC_EMPTY(int b) { return 2 * SB + 2 * SA + 2 + b; }
CEB_DEV int BAR_DRAIN() { return 2 * SB + 2 * SA + 4; }

struct TileInfo {
    int g, ft, row0, rows;
};

CEB_DEV TileInfo decode_tile(const Shared& S, int G, int n_ftiles, int t) {
    int g = 0;
    while (g + 1 < G && t >= S.g_tile[g + 1]) ++g;
    int local = t - S.g_tile[g];
    TileInfo ti;
    ti.g = g;
    ti.ft = local % n_ftiles;
    int tt = local / n_ftiles;
    ti.row0 = S.g_row[g] + tt * BN;
    int rem = S.g_cnt[g] - tt * BN;
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

// dequant prefetch depth (K-blocks in flight per thread of one warpgroup)
template <int FMT>
struct Prefetch {
    static constexpr int depth = FMT == CEB_W_F16 ? 1 : 2;
};

CEB_DEV uint4 ldg128(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

template <int FMT>
CEB_DEV void load_raw(const ceb_wplane& w, int g, int row, int kb, Raw<FMT>& r);

template <>
CEB_DEV void load_raw<CEB_W_Q8_0>(const ceb_wplane& w, int g, int row, int kb, Raw<CEB_W_Q8_0>& r) {
    const size_t grow = (size_t)g * w.n_out + row;
    const uint8_t* q = w.q + grow * w.q_row_bytes + (size_t)kb * 64;
#pragma unroll
    for (int i = 0; i < 4; ++i) r.q[i] = ldg128(q + 16 * i);
    r.sc = __ldg(reinterpret_cast<const uint32_t*>(w.s + grow * w.s_row_bytes + (size_t)kb * 4));
}
template <>
CEB_DEV void load_raw<CEB_W_Q4_K>(const ceb_wplane& w, int g, int row, int kb, Raw<CEB_W_Q4_K>& r) {
    const size_t grow = (size_t)g * w.n_out + row;
    const uint8_t* q = w.q + grow * w.q_row_bytes + (size_t)kb * 32;
    r.q[0] = ldg128(q);
    r.q[1] = ldg128(q + 16);
    r.s = ldg128(w.s + grow * w.s_row_bytes + (size_t)kb * 16);
}
template <>
CEB_DEV void load_raw<CEB_W_F16>(const ceb_wplane& w, int g, int row, int kb, Raw<CEB_W_F16>& r) {
    const size_t grow = (size_t)g * w.n_out + row;
    const uint8_t* q = w.q + grow * w.q_row_bytes + (size_t)kb * 128;
#pragma unroll
    for (int i = 0; i < 8; ++i) r.q[i] = ldg128(q + 16 * i);
}

// ---- conversion into the TMEM A layout: column c holds k = 2c (low half), 2c+1
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
// (|error| <= 1.5e-7 on erf), far below the fp16 rounding of the output.
CEB_DEV float gelu_as(float x) {
    const float z = fabsf(x) * 0.70710678118654752f;
    const float t = __frcp_rn(fmaf(0.3275911f, z, 1.0f));
    float p = fmaf(1.061405429f, t, -1.453152027f);
    p = fmaf(p, t, 1.421413741f);
    p = fmaf(p, t, -0.284496736f);
    p = fmaf(p, t, 0.254829592f);
    p *= t;
    const float e = 1.0f - p * __expf(-z * z);  // erf(|x|/sqrt2)
    const float erf_s = copysignf(e, x);
    return 0.5f * x + 0.5f * x * erf_s;
}

template <int FMT>
__global__ void __launch_bounds__(NTHREADS, 1)
    ceb_gemm_kernel(const __grid_constant__ CUtensorMap tmap, const ceb_wplane w, const ceb_gemm_args a) {
    extern __shared__ uint8_t smem_raw[];
    const Shared S = carve(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = a.offsets ? w.n_groups : 1;
    const int n_ftiles = w.n_out / BM;
    const int nkb = w.k / BK;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NBARS; ++i) {
            uint32_t cnt = 1;
            if (i >= 2 * SB && i < 2 * SB + SA) cnt = 4;                                  // A full: one per dequant warp
            if (i >= 2 * SB + 2 * SA + 2 && i < 2 * SB + 2 * SA + 4) cnt = 4 * EPI_WG;   // acc empty: epilogue warps
            mbar_init(smem_u32(&S.bars[i]), cnt);
        }
        fence_mbar_init();
        *S.abort = 0;
        int tiles = 0;
        for (int g = 0; g < G; ++g) {
            int r0 = a.offsets ? a.offsets[g] : 0;
            int r1 = a.offsets ? a.offsets[g + 1] : a.m_rows;
            if (r0 < 0 || r1 < r0 || r1 > a.m_rows) {
                if (a.err) atomicCAS(a.err, 0, (int)CEB_DEVERR_BAD_GROUP);
                r0 = r1 = 0;
            }
            S.g_tile[g] = tiles;
            S.g_row[g] = r0;
            S.g_cnt[g] = r1 - r0;
            tiles += ((r1 - r0 + BN - 1) / BN) * n_ftiles;
        }
        S.g_tile[G] = tiles;
    }
    if (warp == 0 && lane == 0) tma_prefetch_desc(&tmap);
    if (warp == 1) {
        tmem_alloc(smem_u32(S.tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *S.tmem_slot;
    const int total = S.g_tile[G];
    volatile int* abort = S.abort;
    auto bar = [&](int i) { return smem_u32(&S.bars[i]); };

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                const TileInfo ti = decode_tile(S, G, n_ftiles, t);
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % SB;
                    if (!mbar_wait(bar(BAR_B_EMPTY(s)), ((it / SB) & 1) ^ 1, abort, a.err, CEB_DEVERR_TIMEOUT_TMA)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(bar(BAR_B_FULL(s)), B_STAGE_BYTES);
                    tma_load_2d(smem_u32(S.b_stages + (size_t)s * B_STAGE_BYTES), &tmap, bar(BAR_B_FULL(s)), kb * BK,
                                ti.row0);
                }
            }
            if (!ok) {  // let issued copies land before the CTA can exit
                const uint32_t n = it < SB ? it : SB;
                for (uint32_t i = it - n; i < it; ++i)
                    mbar_wait(bar(BAR_B_FULL(i % SB)), (i / SB) & 1, nullptr, nullptr, 0);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t it = 0, lt = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++lt) {
                const TileInfo ti = decode_tile(S, G, n_ftiles, t);
                const int ab = lt & 1;
                if (!mbar_wait(bar(BAR_ACC_EMPTY(ab)), ((lt >> 1) & 1) ^ 1, abort, a.err, CEB_DEVERR_TIMEOUT_MMA)) break;
                tc_fence_after();
                int n = (ti.rows + 15) & ~15;
                n = n < 16 ? 16 : n;
                const uint32_t idesc = idesc_f16_f32(BM, n);
                const uint32_t d_tmem = tmem + (uint32_t)(ab * BN);
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % SB, sa = it % SA;
                    if (!mbar_wait(bar(BAR_A_FULL(sa)), (it / SA) & 1, abort, a.err, CEB_DEVERR_TIMEOUT_MMA) ||
                        !mbar_wait(bar(BAR_B_FULL(s)), (it / SB) & 1, abort, a.err, CEB_DEVERR_TIMEOUT_MMA)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t bdesc = smem_desc_sw128(smem_u32(S.b_stages + (size_t)s * B_STAGE_BYTES));
                    const uint32_t a_tmem = tmem + (uint32_t)(A_COL0 + sa * 32);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        mma_f16_ts(d_tmem, a_tmem + kk * 8, bdesc + (uint64_t)(kk * 2), idesc, (kb | kk) != 0);
                    mma_commit(bar(BAR_B_EMPTY(s)));
                    mma_commit(bar(BAR_A_EMPTY(sa)));
                }
                if (ok) mma_commit(bar(BAR_ACC_FULL(ab)));
            }
            // every issued MMA has retired before TMEM can be released
            mma_commit(bar(BAR_DRAIN()));
            mbar_wait(bar(BAR_DRAIN()), 0, nullptr, nullptr, 0);
        }
    } else if (warp >= DEQ_WARP0 && warp < EPI_WARP0) {
        // ------------------------------------------------ dequant producers
        const int wg = (warp - DEQ_WARP0) >> 2;  // this warpgroup takes items i with i % DEQ_WG == wg
        const int r = 32 * (warp & 3) + lane;    // weight row within the tile == TMEM lane
        const uint32_t lane_addr = (uint32_t)(32 * (warp & 3)) << 16;
        const int my_tiles = blockIdx.x < total ? (total - 1 - blockIdx.x) / gridDim.x + 1 : 0;
        const int n_items = my_tiles * nkb;
        constexpr int PF = Prefetch<FMT>::depth;
        Raw<FMT> buf[PF];
        auto item_load = [&](int i, Raw<FMT>& dst) {
            const int t = blockIdx.x + (i / nkb) * gridDim.x;
            const TileInfo ti = decode_tile(S, G, n_ftiles, t);
            load_raw<FMT>(w, ti.g, ti.ft * BM + r, i % nkb, dst);
        };
        // own items: i_j = wg + j * DEQ_WG
        const int n_mine = n_items > wg ? (n_items - 1 - wg) / DEQ_WG + 1 : 0;
#pragma unroll
        for (int u = 0; u < PF - 1; ++u)
            if (u < n_mine) item_load(wg + u * DEQ_WG, buf[u]);
        bool ok = true;
        for (int j0 = 0; j0 < n_mine && ok; j0 += PF) {
#pragma unroll
            for (int u = 0; u < PF; ++u) {
                const int j = j0 + u;
                if (j < n_mine && ok) {
                    if (j + PF - 1 < n_mine) item_load(wg + (j + PF - 1) * DEQ_WG, buf[(u + PF - 1) % PF]);
                    const int i = wg + j * DEQ_WG;
                    const int sa = i % SA;
                    const bool got = __all_sync(0xffffffffu, mbar_wait(bar(BAR_A_EMPTY(sa)), ((i / SA) & 1) ^ 1,
                                                                       abort, a.err, CEB_DEVERR_TIMEOUT_DEQ));
                    if (!got) {
                        ok = false;
                    } else {
                        tc_fence_after();
                        uint32_t o[32];
                        convert<FMT>(buf[u], o);
                        tmem_st32(tmem + lane_addr + (uint32_t)(A_COL0 + sa * 32), o);
                        tmem_st_wait();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(bar(BAR_A_FULL(sa)));
                    }
                }
            }
        }
    } else if (warp >= EPI_WARP0) {
        // ------------------------------------------------ epilogue
        const int wg = (warp - EPI_WARP0) >> 2;  // this warpgroup takes 32-column chunks c with c % EPI_WG == wg
        const int r = 32 * (warp & 3) + lane;    // output feature within the tile
        const uint32_t lane_addr = (uint32_t)(32 * (warp & 3)) << 16;
        const bool f16 = (a.epi & CEB_EPI_F16_OUT) != 0, gelu = (a.epi & CEB_EPI_GELU) != 0;
        uint32_t lt = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, ++lt) {
            const TileInfo ti = decode_tile(S, G, n_ftiles, t);
            const int ab = lt & 1;
            if (!__all_sync(0xffffffffu,
                            mbar_wait(bar(BAR_ACC_FULL(ab)), (lt >> 1) & 1, abort, a.err, CEB_DEVERR_TIMEOUT_EPI)))
                break;
            tc_fence_after();
            const int n = ti.ft * BM + r;
            const float bv = (a.epi & CEB_EPI_BIAS) ? a.bias[(size_t)ti.g * a.bias_group_stride + n] : 0.0f;
            for (int c0 = 32 * wg; c0 < ti.rows; c0 += 32 * EPI_WG) {
                uint32_t v[32];
                tmem_ld32(tmem + lane_addr + (uint32_t)(ab * BN + c0), v);
                tmem_ld_wait();
                const int lim = ti.rows - c0 < 32 ? ti.rows - c0 : 32;
                float x[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    x[j] = __uint_as_float(v[j]) + bv;
                    if (gelu) x[j] = gelu_as(x[j]);
                }
                if (f16) {
                    // lane pairs (2i, 2i+1) exchange so each lane stores a half2 of
                    // features (2i, 2i+1): even lanes for even rows, odd lanes for odd rows
                    const bool odd = lane & 1;
                    __half* o = reinterpret_cast<__half*>(a.out) + (size_t)(ti.row0 + c0) * a.ldo + (n & ~1);
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        const float send = odd ? x[j] : x[j + 1];
                        const float got = __shfl_xor_sync(0xffffffffu, send, 1);
                        const int row = odd ? j + 1 : j;
                        const __half2 hv = odd ? __floats2half2_rn(got, x[j + 1]) : __floats2half2_rn(x[j], got);
                        if (row < lim) *reinterpret_cast<__half2*>(o + (size_t)row * a.ldo) = hv;
                    }
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
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

template <int FMT>
int launch_fmt(const CUtensorMap& map, const ceb_wplane& w, const ceb_gemm_args& a, int grid, cudaStream_t st) {
    static bool attr_set = false;
    if (!attr_set) {
        CEB_CUDA_OK(cudaFuncSetAttribute(ceb_gemm_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)SMEM_BYTES));
        attr_set = true;
    }
    ceb_gemm_kernel<FMT><<<grid, NTHREADS, SMEM_BYTES, st>>>(map, w, a);
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
    CUtensorMap map;
    const int mrc = ceb_make_tmap_2d_f16(&map, act_f16, (uint64_t)w.k, (uint64_t)act_rows, (uint64_t)w.k * 2, BK, BN);
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
        case CEB_W_Q8_0: CEB_LAUNCH(CEB_PROF_GEMM, stream, flops, bytes, rc = launch_fmt<CEB_W_Q8_0>(map, w, a, grid, stream)); break;
        case CEB_W_Q4_K: CEB_LAUNCH(CEB_PROF_GEMM, stream, flops, bytes, rc = launch_fmt<CEB_W_Q4_K>(map, w, a, grid, stream)); break;
        case CEB_W_F16: CEB_LAUNCH(CEB_PROF_GEMM, stream, flops, bytes, rc = launch_fmt<CEB_W_F16>(map, w, a, grid, stream)); break;
        default: return ceb_set_error(2, "gemm: unknown weight format %d", w.format);
    }
    return rc;
}
