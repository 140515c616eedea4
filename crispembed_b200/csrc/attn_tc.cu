// attn_tc.cu -- varlen multi-head self-attention on tcgen05 CTA pairs.
//
// Replaces the attention block of the encoder graph (src/crispembed.cpp:1278-1297
// of the reference: softmax(Q K^T / sqrt(head_dim)) V per head over the tokens
// of one sequence, no causal mask) for sequences of up to 512 tokens,
// head_dim 64 and an even head count.  Other shapes use the mma.sync kernel in
// encoder_kernels.cu.
//
// One cluster of 2 CTAs = one (sequence, 256-query tile, pair of heads h, h+1);
// CTA r owns queries q0 + 128 r .. +127 of both heads.  The two heads are two
// independent pipelines through one MMA warp, so the tensor pipe works on one
// head while the other head's softmax runs:
//   S = Q K^T   tcgen05.mma.cta_group::2 (M = 256 = the pair's queries), keys in
//               chunks of 64 (N = 64; each CTA holds 32 keys of a chunk), fp32 S
//               in one of two TMEM buffers per head, so S of chunk c+1 is ready
//               while the softmax of chunk c runs.
//   softmax     one thread per query row, online over the chunks: the row max of
//               the chunk from TMEM, exponentials as fp16 pairs on the MUFU
//               (ex2.approx.f16x2), P written over the chunk's S columns (the S
//               that reuses that buffer is issued after the P V that reads P, and
//               tcgen05 MMAs run in issue order), the row sum as fp16 pair sums
//               widened per chunk.  The max used for the exponentials is raised --
//               and O rescaled in TMEM, after the previous P V -- only when the true
//               max exceeds it by more than 2^2, so exponents stay <= 2 and P <= 4.
//               Without a rescale P is published at once, ahead of the wait for
//               the previous chunk's P V (per-buffer barriers keep that wait from
//               ever running two phases behind).
//   O = P V     TS form: A = P from TMEM, B = V MN-major (64-byte swizzle), each
//               CTA holding 32 of the 64 dims for all keys; O (fp32) in TMEM,
//               divided by the row sum at the end and stored fp16.
// TMEM per CTA: head A  S/P buffers 0..63 and 64..127, O 128..191; head B +256.
// Barriers that a waiter could otherwise find two phases ahead (S, P, P V) exist once
// per buffer.
// Rank 1's "P written" is relayed to the leader's barrier by a 16-byte
// cp.async.bulk (asynchronous; a blocking cluster-scope release arrive costs
// ~1500 cycles).  The kernel uses more than half of the SM's shared memory, so
// each CTA is alone on its SM and holds all 512 TMEM columns.  Every wait is
// bounded and reports through the error word.
#include "ceb_encoder_internal.h"
#include "ceb_internal.h"
#include "common.cuh"

namespace {

constexpr int HD = 64;            // head dim
constexpr int QT = 128;           // queries per CTA (MMA M = 256 per pair)
constexpr int LMAX = 512;         // longest sequence handled here
constexpr int KC = 64;            // keys per chunk (S MMA N)
constexpr int NCH = LMAX / KC;    // max chunks
constexpr int Q_BYTES = QT * HD * 2;                 // 16 KB
constexpr int KH_BYTES = (KC / 2) * HD * 2;          // 4 KB: this CTA's 32 keys of one chunk
constexpr int K_BYTES = NCH * KH_BYTES;              // 32 KB
constexpr int VB_KEYS = 128;                         // keys per V box
constexpr int VB_BYTES = VB_KEYS * 32 * 2;           // 8 KB: 128 keys x this CTA's 32 dims
constexpr int V_BYTES = (LMAX / VB_KEYS) * VB_BYTES; // 32 KB
constexpr int HEAD_BYTES = Q_BYTES + K_BYTES + V_BYTES;  // 80 KB per head
constexpr uint32_t BUF_STRIDE = 64;                    // S/P buffer b at columns 64 b
constexpr uint32_t O_COL = 128, HEAD_COLS = 256;
#ifndef CEB_ATTN_RESCALE_LOG2
#define CEB_ATTN_RESCALE_LOG2 2.0f
#endif
// raise the exponent's max when exceeded by more than 2^2: exponents stay <= 2, so their
// fp16 rounding (the exponentials are taken in fp16 pairs) costs at most 2^-11 relative
constexpr float RESCALE_LOG2 = CEB_ATTN_RESCALE_LOG2;
constexpr int SBUF = 2;                                // S/P buffers per head
#ifndef CEB_ATTN_HPC
#define CEB_ATTN_HPC 1
#endif
constexpr int HPC = CEB_ATTN_HPC;  // heads per CTA pair (interleaved through one MMA warp)
constexpr int NTHR = 128 + 128 * HPC;  // warps 0 TMA, 1 TMEM+MMA, 2..3 relays, 4.. softmax (4 per head)
constexpr int SM_WARP0 = 4;
// barriers, per head h: +h*PER; S, P and PLOCAL once per S/P buffer (+b)
enum { B_LDQK, B_LDV, B_S, B_S1, B_P, B_P1, B_PV, B_PV1, B_PLOCAL, B_PLOCAL1, PER };
constexpr int B_DRAIN = HPC * PER, NBAR = HPC * PER + 1;
// two heads: ~161 KB, one CTA per SM (512 TMEM columns); one head: ~81 KB, at most two CTAs
// per SM (256 columns each), so TMEM allocations never wait on one another
constexpr size_t SMEM_LAUNCH = 1024 + HPC * HEAD_BYTES + 256;
constexpr uint32_t TMEM_ALLOC = 256 * HPC;
static_assert(HPC == 1 || HPC == 2, "heads per CTA");
static_assert(HPC == 2 || 3 * SMEM_LAUNCH > 228 * 1024, "at most two one-head CTAs per SM");
static_assert(NBAR * 8 <= 192, "barrier area");
static_assert(SMEM_LAUNCH <= 227 * 1024, "attention shared memory");

CEB_DEV float ex2f(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
// 2^t0, 2^t1 as the packed fp16 pair P is stored in: one conversion, one MUFU op
CEB_DEV uint32_t ex2_h2(float t0, float t1) {
    uint32_t in = h2_as_u32(__floats2half2_rn(t0, t1)), r;
    asm("ex2.approx.f16x2 %0, %1;" : "=r"(r) : "r"(in));
    return r;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NTHR, 1)
    attn_pair_kernel(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap k_map,
                     const __grid_constant__ CUtensorMap v_map, const int32_t* __restrict__ cu, int d, float scale_log2,
                     __half* __restrict__ out, int* err, int total_rows, int max_len) {
    const int seq = blockIdx.z, head0 = HPC * blockIdx.y;
    const int start = cu[seq], len = cu[seq + 1] - start;
    // row offsets that leave the rows or disagree with max_len: report, touch nothing
    // (both CTAs of the pair read the same offsets and return together)
    if (start < 0 || len < 0 || len > total_rows - start || len > max_len) {
        if (blockIdx.x == 0 && head0 == 0 && threadIdx.x == 0 && err) atomicCAS(err, 0, (int)CEB_DEVERR_BAD_INDEX);
        return;
    }
    const int q0 = (blockIdx.x >> 1) * 2 * QT;
    if (q0 >= len || len > LMAX) return;  // both CTAs of the pair take the same branch

    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    auto sQ = [&](int h) { return base + h * HEAD_BYTES; };
    auto sK = [&](int h) { return base + h * HEAD_BYTES + Q_BYTES; };
    auto sV = [&](int h) { return base + h * HEAD_BYTES + Q_BYTES + K_BYTES; };
    uint8_t* misc = base + HPC * HEAD_BYTES;               // 1024-byte aligned
    uint64_t* bars = reinterpret_cast<uint64_t*>(misc);    // <= 192 bytes
    uint8_t* sig = misc + 192;                             // 2 x 16 bytes: sinks (leader) / sources (rank 1)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 224);
    int* abort_flag = reinterpret_cast<int*>(misc + 228);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int lpad = (len + 31) & ~31;                     // keys as the MMAs see them
    const int nch = (lpad + KC - 1) / KC;
    const int n_vb = (lpad + VB_KEYS - 1) / VB_KEYS;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NBAR; ++i) {
            const int r = i % PER;
            const bool four = r == B_P || r == B_P1 || r == B_PLOCAL || r == B_PLOCAL1;
            mbar_init(smem_u32(&bars[i]), (i < HPC * PER && four) ? 4 : 1);
        }
        fence_mbar_init();
        *abort_flag = 0;
        *reinterpret_cast<uint4*>(sig) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(sig + 16) = make_uint4(0, 0, 0, 0);
        fence_proxy_async_smem();
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_slot), TMEM_ALLOC);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    volatile int* abort = abort_flag;
    auto bar = [&](int i) { return smem_u32(&bars[i]); };
    auto lead_bar = [&](int i) { return mapa_shared(bar(i), 0); };
    auto wait_at = [&](int i, uint32_t par, int code) {
        return mbar_wait(bar(i), par, abort, err, code | ((i + 1) << 16));
    };
    auto wait_cl = [&](int i, uint32_t par, int code) {
        return mbar_wait_cluster(bar(i), par, abort, err, code | ((i + 1) << 16));
    };

    if (warp == 0) {
        // ------------------------------------------------ TMA: per head Q, this CTA's key halves, its V dims
        if (lane == 0) {
            for (int h = 0; h < HPC; ++h) {
                const int hd = head0 + h;
                if (leader) {
                    mbar_arrive_expect_tx(bar(h * PER + B_LDQK), 2u * (Q_BYTES + nch * KH_BYTES));
                    mbar_arrive_expect_tx(bar(h * PER + B_LDV), 2u * n_vb * VB_BYTES);
                }
                tma_load_2d_pair(smem_u32(sQ(h)), &q_map, lead_bar(h * PER + B_LDQK), hd * HD,
                                 start + q0 + QT * (int)rank);
                for (int c = 0; c < nch; ++c) {
                    const int nc = min(KC, lpad - c * KC);
                    tma_load_2d_pair(smem_u32(sK(h) + c * KH_BYTES), &k_map, lead_bar(h * PER + B_LDQK), d + hd * HD,
                                     start + c * KC + (int)rank * (nc / 2));
                }
                for (int vb = 0; vb < n_vb; ++vb)
                    tma_load_2d_pair(smem_u32(sV(h) + vb * VB_BYTES), &v_map, lead_bar(h * PER + B_LDV),
                                     2 * d + hd * HD + 32 * (int)rank, start + vb * VB_KEYS);
            }
            if (leader)  // the pair's copies have landed before this CTA can exit
                for (int h = 0; h < HPC; ++h) {
                    mbar_wait_cluster(bar(h * PER + B_LDQK), 0, nullptr, nullptr, 0);
                    mbar_wait_cluster(bar(h * PER + B_LDV), 0, nullptr, nullptr, 0);
                }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer (leader): S and P V of both heads, interleaved
        if (leader && lane == 0) {
            const uint32_t pv_idesc = idesc_f16_f32(2 * QT, HD) | (1u << 16);  // B (V) MN-major
            auto issue_s = [&](int h, int c) {
                const int nc = min(KC, lpad - c * KC), b = SBUF == 2 ? (c & 1) : 0;
                const uint64_t qdesc = smem_desc_sw128(smem_u32(sQ(h)));
                const uint64_t kdesc = smem_desc_sw128(smem_u32(sK(h) + c * KH_BYTES));
                const uint32_t idesc = idesc_f16_f32(2 * QT, nc);
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk)
                    mma_pair_f16_ss(tmem + h * HEAD_COLS + BUF_STRIDE * (uint32_t)b, qdesc + (uint64_t)(kk * 2),
                                    kdesc + (uint64_t)(kk * 2), idesc, kk != 0);
                mma_pair_commit(bar(h * PER + B_S + b));
                mma_pair_commit(mapa_shared(bar(h * PER + B_S + b), 1));
            };
            bool ok = true;
            for (int h = 0; h < HPC && ok; ++h) ok = wait_cl(h * PER + B_LDQK, 0, CEB_DEVERR_TIMEOUT_MMA);
            if (ok) {
                tc_fence_after();
                for (int c = 0; c < SBUF && c < nch; ++c)
                    for (int h = 0; h < HPC; ++h) issue_s(h, c);
            }
            for (int c = 0; c < nch && ok; ++c) {
                const int b = SBUF == 2 ? (c & 1) : 0;
                const uint32_t pp = SBUF == 2 ? (c >> 1) & 1 : c & 1;
                for (int h = 0; h < HPC && ok; ++h) {
                    ok = wait_cl(h * PER + B_P + b, pp, CEB_DEVERR_TIMEOUT_MMA) &&
                         (c > 0 || wait_cl(h * PER + B_LDV, 0, CEB_DEVERR_TIMEOUT_MMA));
                    if (!ok) break;
                    tc_fence_after();
                    const int nc = min(KC, lpad - c * KC);
                    const uint64_t vdesc = smem_desc_mn_sw64(smem_u32(sV(h))) + (uint64_t)(c * KC * 4);  // 64 B per key
                    for (int j = 0; j < nc / 16; ++j)
                        mma_pair_f16_ts(tmem + h * HEAD_COLS + O_COL,
                                        tmem + h * HEAD_COLS + BUF_STRIDE * (uint32_t)b + (uint32_t)(8 * j), vdesc + (uint64_t)(64 * j),
                                        pv_idesc, (c | j) != 0);
                    mma_pair_commit(bar(h * PER + B_PV + b));
                    mma_pair_commit(mapa_shared(bar(h * PER + B_PV + b), 1));
                    if (c + SBUF < nch) issue_s(h, c + SBUF);  // reuses buffer b after the P V that reads it
                }
            }
            mma_pair_commit(bar(B_DRAIN));
            mbar_wait(bar(B_DRAIN), 0, nullptr, nullptr, 0);
        }
    } else if (warp == 2 || warp == 3) {
        // ------------------------------------------------ relays (rank 1): head (warp-2)'s P written -> leader
        const int h = warp - 2;
        if (h < HPC && !leader && lane == 0) {
            for (int c = 0; c < nch; ++c) {
                const int b = SBUF == 2 ? (c & 1) : 0;
                if (!wait_at(h * PER + B_PLOCAL + b, SBUF == 2 ? (c >> 1) & 1 : c & 1, CEB_DEVERR_TIMEOUT_EPI)) break;
                bulk_copy_to_cluster(mapa_shared(smem_u32(sig + 16 * h), 0), smem_u32(sig + 16 * h), 16,
                                     lead_bar(h * PER + B_P + b));
            }
        }
    } else if (warp >= SM_WARP0) {
        // ------------------------------------------------ softmax + output, thread = query row of head h
        const int h = (warp - SM_WARP0) >> 2;
        const int qd = warp & 3;                                // TMEM lane quadrant
        const uint32_t row_t = tmem + ((uint32_t)(32 * qd) << 16) + h * HEAD_COLS;
        const int q = q0 + QT * (int)rank + 32 * qd + lane;     // query index within the sequence
        float m_use = -INFINITY;  // max used by the exponentials (log2 units)
        float l_run = 0.0f;       // row sum of P (fp16 pair sums widened per chunk)
        bool ok = true;
        for (int c = 0; c < nch; ++c) {
            const int k0 = c * KC, nc = min(KC, lpad - k0), b = SBUF == 2 ? (c & 1) : 0;
            const uint32_t pp = SBUF == 2 ? (c >> 1) & 1 : c & 1;
            const uint32_t buf = row_t + BUF_STRIDE * (uint32_t)b;
            ok = __all_sync(0xffffffffu, wait_at(h * PER + B_S + b, pp, CEB_DEVERR_TIMEOUT_EPI));
            if (!ok) break;
            tc_fence_after();
            uint32_t v[2][32];
            tmem_ld32(buf, v[0]);
            if (nc > 32) tmem_ld32(buf + 32, v[1]);
            tmem_ld_wait();
            if (k0 + nc > len) {  // the sequence ends in this chunk (same for every thread): no weight past it
#pragma unroll
                for (int g = 0; g < 2; ++g)
#pragma unroll
                    for (int t = 0; t < 32; ++t)
                        if (k0 + 32 * g + t >= len) v[g][t] = 0xff800000u;  // -inf
            }
            float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int t = 0; t < 32; ++t) mx[t & 3] = fmaxf(mx[t & 3], __uint_as_float(v[0][t]));
            if (nc > 32) {
#pragma unroll
                for (int t = 0; t < 32; ++t) mx[t & 3] = fmaxf(mx[t & 3], __uint_as_float(v[1][t]));
            }
            const float cm = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * scale_log2;
            // raise the max used by the exponentials when the true max exceeds it by more than
            // 2^RESCALE_LOG2 (always on the first chunk: m_use = -inf); warp-uniform decision
            const bool raise = c > 0 && __any_sync(0xffffffffu, cm > m_use + RESCALE_LOG2);
            float alpha = 1.0f;
            if (c == 0) {
                m_use = cm;
            } else if (raise) {
                const float m_new = fmaxf(m_use, cm);
                alpha = ex2f(m_use - m_new);
                m_use = m_new;
            }
            // P = 2^(s*scale - m) as fp16 pairs over the S columns just read; the row sum adds
            // the pairs in fp16 (a 16-pair tree per 32 keys, values <= 4) and widens per chunk
            const float nm = -m_use;
            float csum = 0.0f;
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                if (32 * g < nc) {
                    uint32_t pk[16];
#pragma unroll
                    for (int t = 0; t < 32; t += 2)
                        pk[t >> 1] = ex2_h2(fmaf(__uint_as_float(v[g][t]), scale_log2, nm),
                                            fmaf(__uint_as_float(v[g][t + 1]), scale_log2, nm));
                    tmem_st16(buf + (uint32_t)(16 * g), pk);
                    __half2 a[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) a[i] = __hadd2(u32_as_h2(pk[2 * i]), u32_as_h2(pk[2 * i + 1]));
#pragma unroll
                    for (int w = 4; w >= 1; w >>= 1)
#pragma unroll
                        for (int i = 0; i < w; ++i) a[i] = __hadd2(a[i], a[i + w]);
                    csum += __low2float(a[0]) + __high2float(a[0]);
                }
            }
            l_run = l_run * alpha + csum;
            auto publish = [&]() {
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if (!leader)
                        mbar_arrive(bar(h * PER + B_PLOCAL + b));
                    else if (qd == 0)
                        mbar_arrive_expect_tx(bar(h * PER + B_P + b), 16);  // + rank 1's relayed signal
                    else
                        mbar_arrive(bar(h * PER + B_P + b));
                }
            };
            // Without a rescale P of chunk c is published at once (P V of chunk c runs after that
            // of c-1 in issue order); a rescale of O waits for P V of chunk c-1 first.
            const bool pub_now = !raise;
            if (pub_now) publish();
            if (c > 0) {
                // per-parity barriers: the next phase of this one needs P of chunk c+1
                const int cp = c - 1;
                ok = __all_sync(0xffffffffu,
                                wait_at(h * PER + B_PV + (cp & 1), (cp >> 1) & 1, CEB_DEVERR_TIMEOUT_EPI));
                if (!ok) break;
                if (raise) {
                    tc_fence_after();
#pragma unroll
                    for (int o0 = 0; o0 < HD; o0 += 32) {
                        uint32_t ov[32];
                        tmem_ld32(row_t + O_COL + (uint32_t)o0, ov);
                        tmem_ld_wait();
#pragma unroll
                        for (int t = 0; t < 32; ++t) ov[t] = __float_as_uint(__uint_as_float(ov[t]) * alpha);
                        tmem_st32(row_t + O_COL + (uint32_t)o0, ov);
                    }
                }
            }
            if (!pub_now) publish();
        }
        const int cl = nch - 1;
        if (ok && __all_sync(0xffffffffu,
                             wait_at(h * PER + B_PV + (cl & 1), (cl >> 1) & 1, CEB_DEVERR_TIMEOUT_EPI))) {
            tc_fence_after();
            const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
            uint32_t pk[32];
#pragma unroll
            for (int o0 = 0; o0 < HD; o0 += 32) {
                uint32_t v[32];
                tmem_ld32(row_t + O_COL + (uint32_t)o0, v);
                tmem_ld_wait();
#pragma unroll
                for (int t = 0; t < 32; t += 2)
                    pk[(o0 + t) >> 1] =
                        h2_as_u32(__floats2half2_rn(__uint_as_float(v[t]) * inv, __uint_as_float(v[t + 1]) * inv));
            }
            if (q < len) {
                uint4* o = reinterpret_cast<uint4*>(out + (size_t)(start + q) * d + (head0 + h) * HD);
#pragma unroll
                for (int c = 0; c < 8; ++c) o[c] = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
            }
        }
    }

    tc_fence_before();
    __syncwarp();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, TMEM_ALLOC);
    }
}


}  // namespace

// Returns 1 (nothing launched) when the shape is not handled here.
int ceb_attention_tc(const __half* qkv, int total_rows, const int32_t* cu, int n_seqs, int max_len, int d, int n_head,
                     __half* out, int* d_err, cudaStream_t st) {
    if (n_head <= 0 || (n_head % HPC) || d != n_head * HD || max_len > LMAX || max_len <= 0) return 1;
    if ((reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) return 1;
    if (int rc = ceb_func_smem(reinterpret_cast<const void*>(attn_pair_kernel), SMEM_LAUNCH)) return rc;
    CUtensorMap q_map, k_map, v_map;
    const uint64_t ld_bytes = (uint64_t)3 * d * 2;
    int rc = ceb_make_tmap_2d_sw(&q_map, qkv, 2, (uint64_t)3 * d, (uint64_t)total_rows, ld_bytes, HD, QT, 128);
    if (rc) return rc;
    rc = ceb_make_tmap_2d_sw(&k_map, qkv, 2, (uint64_t)3 * d, (uint64_t)total_rows, ld_bytes, HD, KC / 2, 128);  // 32 keys
    if (rc) return rc;
    rc = ceb_make_tmap_2d_sw(&v_map, qkv, 2, (uint64_t)3 * d, (uint64_t)total_rows, ld_bytes, 32, VB_KEYS, 64);
    if (rc) return rc;
    const float scale_log2 = (1.0f / sqrtf((float)HD)) * 1.4426950408889634f;
    const int n_qpairs = (max_len + 2 * QT - 1) / (2 * QT);
    dim3 grid(2 * n_qpairs, n_head / HPC, n_seqs);
    CEB_LAUNCH(CEB_PROF_ATTN, st, 0.0, 0.0,
               attn_pair_kernel<<<grid, NTHR, SMEM_LAUNCH, st>>>(q_map, k_map, v_map, cu, d, scale_log2, out, d_err,
                                                                  total_rows, max_len));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}
