// attn_fa.cu -- varlen multi-head self-attention on single-CTA tcgen05 MMAs.
//
// Replaces the attention block of the encoder graph (src/crispembed.cpp:1278-1297
// of the reference: softmax(Q K^T / sqrt(head_dim)) V per head over the tokens of
// one sequence, no causal mask) for head_dim 64 and any sequence length.
//
// Persistent CTAs (two per SM) take items = (sequence, head, 128-query tile) from a
// device counter, so a CTA that drew short items draws more (the last CTA to finish
// returns the counter to zero for the next launch); the TMA warp hands each item index
// to the other roles through a small ring in shared memory, loads the next item's Q (two
// Q buffers) and first K / V chunks while the current item finishes, and every barrier
// phase follows one chunk counter that runs across the items of a CTA.  Keys stream in
// chunks of 128:
//   S = Q K^T   tcgen05.mma.cta_group::1, M = 128 queries, N = 128 keys, fp32 S in
//               TMEM; Q and the K chunk by TMA (128-byte swizzle, K-major).
//   softmax     one thread per query row (4 warps, one per TMEM lane quadrant):
//               the chunk's S row into registers with one wait, its max, then
//               exponentials as fp16 pairs (ex2.approx.f16x2).  Once S is read the
//               next S may be issued (it overlaps the exponentials); P goes to its own TMEM
//               columns after the previous chunk's P V has finished reading them.
//               The max used for the exponentials is raised -- and O rescaled in
//               TMEM -- only when the true max exceeds it by more than 2^2, so
//               exponents stay <= 2 and P <= 4.  Row sums as fp16 pair sums
//               widened to fp32 per chunk.  No exponentials for 32-key pieces past
//               the sequence (P = 0 there) or for warps whose rows all lie past it.
//   O = P V     TS form: A = P from TMEM, B = the V chunk MN-major (the same
//               128-byte-swizzled TMA image as K), O (fp32) in TMEM; divided by
//               the row sum at the end and stored fp16.
// TMEM: S columns 0..127, P 128..191, O 192..255.  Two CTAs per SM (99 KB of
// shared memory each): a CTA's MMAs issue one at a time with ~115 cycles of latency
// each, so the two CTAs' MMA streams and softmaxes interleave on the tensor pipe.
// The next item's first P V (accumulate off) is issued only after its first P,
// which the softmax warps write after they have read the previous item's O.
// Every barrier completes once per chunk and is waited on once per chunk, in
// order, by a role that the next completion depends on (no phase can be
// skipped).  Every wait is bounded and reports through the error word.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "ceb_encoder_internal.h"
#include "ceb_internal.h"
#include "common.cuh"

namespace {

constexpr int HD = 64;                         // head dim
constexpr int QT = 128;                        // queries per CTA (MMA M)
constexpr int KC = 128;                        // keys per chunk (S MMA N)
constexpr int NS = 2;                          // K/V stages
constexpr int TILE_BYTES = 128 * HD * 2;       // 16 KB: 128 rows of 64 fp16, 128-byte swizzle
constexpr int STAGE_BYTES = 2 * TILE_BYTES;    // K and V of one chunk
constexpr uint32_t S_COL = 0, P_COL = 128, O_COL = 192, TMEM_COLS = 256;
constexpr int NTHR = 192;                      // warp 0 TMA, warp 1 TMEM + MMA, warps 2..5 softmax
constexpr int CTAS_PER_SM = 2;
constexpr int NRING = 4;  // item indices handed from the TMA warp to the other roles
enum { B_QFULL, B_QFREE = B_QFULL + 2, B_FULL = B_QFREE + 2, B_EMPTY = B_FULL + NS, B_SFULL = B_EMPTY + NS, B_SFREE,
       B_PFULL, B_PVDONE, B_DRAIN, B_IFULL, B_IEMPTY = B_IFULL + NRING, NBAR = B_IEMPTY + NRING };
constexpr size_t SMEM_LAUNCH = 1024 + 2 * TILE_BYTES + NS * STAGE_BYTES + 256;
static_assert(NBAR * 8 + 8 + 4 * NRING <= 256, "barrier area");
static_assert(3 * SMEM_LAUNCH > 228 * 1024, "at most two CTAs per SM (256 TMEM columns each)");
#ifndef CEB_FA_RESCALE_LOG2
#define CEB_FA_RESCALE_LOG2 2.0f
#endif
constexpr float RESCALE_LOG2 = CEB_FA_RESCALE_LOG2;

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
// MN-major operand, 128-byte swizzle: rows of 128 B (64 fp16 along N) consecutive
// along K, 8-row (1024 B) swizzle atoms; one atom along N.
CEB_DEV uint64_t smem_desc_mn_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFF) >> 4);  // start address  [0,14)
    d |= (uint64_t)1 << 16;                   // leading byte offset (single atom along N)
    d |= (uint64_t)(1024 >> 4) << 32;         // stride byte offset: next 8 K-rows
    d |= (uint64_t)1 << 46;                   // descriptor version (sm100)
    d |= (uint64_t)2 << 61;                   // SWIZZLE_128B
    return d;
}

struct Item {
    int head, q0, start, len;
};
// Item i -> (query tile, head, sequence), the query tile fastest so that the items of
// one (sequence, head) are taken side by side and share K / V in L2.  False for an
// empty item (query tile past the sequence) and for bad row offsets (reported when
// err is given).
CEB_DEV bool decode_item(int i, int n_qt, int n_head, const int32_t* __restrict__ cu, int total_rows, int max_len,
                         int* err, Item& it) {
    const int qt = i % n_qt, rest = i / n_qt;
    const int seq = rest / n_head;
    it.head = rest - seq * n_head;
    it.start = cu[seq];
    it.len = cu[seq + 1] - it.start;
    it.q0 = qt * QT;
    if (it.start < 0 || it.len < 0 || it.len > total_rows - it.start || it.len > max_len) {
        if (qt == 0 && it.head == 0 && err) atomicCAS(err, 0, (int)CEB_DEVERR_BAD_INDEX);
        return false;
    }
    return it.q0 < it.len;
}

__global__ void __launch_bounds__(NTHR, CTAS_PER_SM)
    attn_fa_kernel(const __grid_constant__ CUtensorMap map, const int32_t* __restrict__ cu, int n_items, int n_qt,
                   int n_head, int d, float scale_log2, __half* __restrict__ out, int* err, int total_rows,
                   int max_len, int* __restrict__ sched) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = base;                    // two Q buffers (items alternate)
    uint8_t* sKV = base + 2 * TILE_BYTES;  // stage s: K at s * STAGE_BYTES, V TILE_BYTES after it
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + 2 * TILE_BYTES + NS * STAGE_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBAR);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
    volatile int* ring = reinterpret_cast<volatile int*>(abort_flag + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NBAR; ++i)
            mbar_init(smem_u32(&bars[i]), (i == B_SFREE || i == B_PFULL) ? 4 : (i >= B_IEMPTY ? 5 : 1));
        fence_mbar_init();
        *abort_flag = 0;
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    volatile int* abort = abort_flag;
    auto bar = [&](int i) { return smem_u32(&bars[i]); };
    auto wait_at = [&](int i, uint32_t par, int code) {
        return mbar_wait(bar(i), par, abort, err, code | ((i + 1) << 16));
    };
    // The consumers' view of the item stream: the n-th item index from the ring, -1 at the
    // end (or false on abort); every consumer role (MMA lane, 4 softmax warps) releases the slot.
    auto next_item = [&](int n, int code, bool warp_wide, int& idx) {
        const int r = n % NRING;
        bool ok = mbar_wait(bar(B_IFULL + r), (n / NRING) & 1, abort, err, code | ((B_IFULL + r + 1) << 16));
        if (warp_wide) ok = __all_sync(0xffffffffu, ok);
        if (!ok) return false;
        idx = ring[r];
        if (warp_wide) __syncwarp();
        if (!warp_wide || lane == 0) mbar_arrive(bar(B_IEMPTY + r));
        return true;
    };

    if (warp == 0) {
        // ------------------------------------------------ TMA: per item Q, then K and V per chunk
        if (lane == 0) {
            int g = 0, n_it = 0;  // chunks and items issued
            bool ok = true;
            // hand item index v to the other roles through ring slot n_it % NRING
            auto publish = [&](int v) {
                const int r = n_it % NRING;
                if (n_it >= NRING && !wait_at(B_IEMPTY + r, ((n_it / NRING) - 1) & 1, CEB_DEVERR_TIMEOUT_TMA))
                    return false;
                ring[r] = v;
                mbar_arrive(bar(B_IFULL + r));  // release: the index is visible to the waiters
                return true;
            };
            while (ok) {
                // items are taken dynamically: a CTA that drew short items draws more
                const int i = atomicAdd(sched, 1);
                if (i >= n_items) break;
                Item it;
                if (!decode_item(i, n_qt, n_head, cu, total_rows, max_len, err, it)) continue;
                const int qb = n_it & 1;
                if ((n_it >= 2 && !wait_at(B_QFREE + qb, ((n_it >> 1) - 1) & 1, CEB_DEVERR_TIMEOUT_TMA)) ||
                    !publish(i)) {
                    ok = false;
                    break;
                }
                const int col_q = it.head * HD, col_k = d + it.head * HD, col_v = 2 * d + it.head * HD;
                mbar_arrive_expect_tx(bar(B_QFULL + qb), TILE_BYTES);
                tma_load_2d(smem_u32(sQ + qb * TILE_BYTES), &map, bar(B_QFULL + qb), col_q, it.start + it.q0);
                ++n_it;
                const int nch = (it.len + KC - 1) / KC;
                for (int c = 0; c < nch; ++c, ++g) {
                    const int s = g % NS;
                    if (g >= NS && !wait_at(B_EMPTY + s, ((g / NS) - 1) & 1, CEB_DEVERR_TIMEOUT_TMA)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(bar(B_FULL + s), STAGE_BYTES);
                    tma_load_2d(smem_u32(sKV + s * STAGE_BYTES), &map, bar(B_FULL + s), col_k, it.start + c * KC);
                    tma_load_2d(smem_u32(sKV + s * STAGE_BYTES + TILE_BYTES), &map, bar(B_FULL + s), col_v,
                                it.start + c * KC);
                }
            }
            if (ok) publish(-1);  // end of the stream (on abort the consumers leave on the flag)
            // the scheduling counter returns to 0 for the next launch once every CTA has drawn
            // its last item: the last CTA to get here resets it
            __threadfence();
            if (atomicAdd(sched + 1, 1) == (int)gridDim.x - 1) {
                atomicExch(sched, 0);
                atomicExch(sched + 1, 0);
            }
            // every copy in flight lands before the CTA can exit (earlier ones were consumed)
            for (int k = n_it > 2 ? n_it - 2 : 0; k < n_it; ++k)
                mbar_wait(bar(B_QFULL + (k & 1)), (k >> 1) & 1, nullptr, nullptr, 0);
            for (int c = g > NS ? g - NS : 0; c < g; ++c)
                mbar_wait(bar(B_FULL + c % NS), (c / NS) & 1, nullptr, nullptr, 0);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer: S(g), then P V of chunk g-1
        if (lane == 0) {
            const uint32_t s_idesc = idesc_f16_f32(QT, KC);
            const uint32_t pv_idesc = idesc_f16_f32(QT, HD) | (1u << 16);  // B (V) MN-major
            int g = 0, n_it = 0;
            bool prev_first = false;  // chunk g-1 was the first chunk of its item (P V overwrites O)
            bool ok = true;
            auto issue_pv = [&](int gp, bool first) {
                const int sp = gp % NS;
                if (!wait_at(B_PFULL, gp & 1, CEB_DEVERR_TIMEOUT_MMA)) return false;
                tc_fence_after();
                const uint64_t vdesc = smem_desc_mn_sw128(smem_u32(sKV + sp * STAGE_BYTES + TILE_BYTES));
#pragma unroll
                for (int j = 0; j < KC / 16; ++j)  // 16 keys = 2048 B of V, 8 TMEM columns of P
                    mma_f16_ts(tmem + O_COL, tmem + P_COL + (uint32_t)(8 * j), vdesc + (uint64_t)(128 * j), pv_idesc,
                               !(first && j == 0));
                mma_commit(bar(B_PVDONE));
                mma_commit(bar(B_EMPTY + sp));
                return true;
            };
            for (;;) {
                int idx = -1;
                if (!(ok = next_item(n_it, CEB_DEVERR_TIMEOUT_MMA, false, idx)) || idx < 0) break;
                Item it;
                decode_item(idx, n_qt, n_head, cu, total_rows, max_len, nullptr, it);
                const int qb = n_it & 1;
                if (!(ok = wait_at(B_QFULL + qb, (n_it >> 1) & 1, CEB_DEVERR_TIMEOUT_MMA))) break;
                ++n_it;
                const uint64_t qdesc = smem_desc_sw128(smem_u32(sQ + qb * TILE_BYTES));
                const int nch = (it.len + KC - 1) / KC;
                for (int c = 0; c < nch; ++c, ++g) {
                    const int s = g % NS;
                    ok = wait_at(B_FULL + s, (g / NS) & 1, CEB_DEVERR_TIMEOUT_MMA) &&
                         (g == 0 || wait_at(B_SFREE, (g - 1) & 1, CEB_DEVERR_TIMEOUT_MMA));
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t kdesc = smem_desc_sw128(smem_u32(sKV + s * STAGE_BYTES));
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk)
                        mma_f16_ss(tmem + S_COL, qdesc + (uint64_t)(2 * kk), kdesc + (uint64_t)(2 * kk), s_idesc, kk != 0);
                    mma_commit(bar(B_SFULL));
                    if (c == nch - 1) mma_commit(bar(B_QFREE + qb));  // the item's last S has read Q
                    if (g > 0 && !(ok = issue_pv(g - 1, prev_first))) break;
                    prev_first = c == 0;
                }
                if (!ok) break;
            }
            if (ok && g > 0) issue_pv(g - 1, prev_first);
            mma_commit(bar(B_DRAIN));  // every MMA issued has finished before TMEM is freed
            mbar_wait(bar(B_DRAIN), 0, nullptr, nullptr, 0);
        }
    } else {
        // ------------------------------------------------ softmax + output, thread = query row
        const int qd = warp & 3;  // TMEM lane quadrant of this warp
        const uint32_t row_t = tmem + ((uint32_t)(32 * qd) << 16);
        int g = 0, n_it = 0;
        bool ok = true;
        for (;;) {
            int idx = -1;
            if (!(ok = next_item(n_it++, CEB_DEVERR_TIMEOUT_EPI, true, idx)) || idx < 0) break;
            Item it;
            decode_item(idx, n_qt, n_head, cu, total_rows, max_len, nullptr, it);
            const int len = it.len, nch = (len + KC - 1) / KC;
            // a warp whose 32 query rows all lie past the sequence keeps to the barrier protocol but
            // computes no exponentials (its P rows stay stale; they only reach O rows never stored)
            const bool dead = it.q0 + 32 * qd >= len;
            float m_use = -INFINITY, l_run = 0.0f;  // max used by the exponentials (log2 units), row sum
            for (int c = 0; c < nch; ++c, ++g) {
                ok = __all_sync(0xffffffffu, wait_at(B_SFULL, g & 1, CEB_DEVERR_TIMEOUT_EPI));
                if (!ok) break;
                tc_fence_after();
                const int k0 = c * KC;
                const bool tail = k0 + KC > len;  // the sequence ends in this chunk: no weight past it
                const int nv = tail ? (len - k0 + 31) / 32 : KC / 32;  // 32-key pieces holding a key
                // the chunk's S row in registers with one wait; then S may be overwritten by the next chunk
                uint32_t v[KC / 32][32];
#pragma unroll
                for (int pc = 0; pc < KC / 32; ++pc) tmem_ld32(row_t + S_COL + (uint32_t)(32 * pc), v[pc]);
                tmem_ld_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(B_SFREE));
                if (tail) {
#pragma unroll
                    for (int pc = 0; pc < KC / 32; ++pc)
#pragma unroll
                        for (int t = 0; t < 32; ++t)
                            if (k0 + 32 * pc + t >= len) v[pc][t] = 0xff800000u;  // -inf
                }
                float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int pc = 0; pc < KC / 32; ++pc)
#pragma unroll
                    for (int t = 0; t < 32; ++t) mx[t & 3] = fmaxf(mx[t & 3], __uint_as_float(v[pc][t]));
                const float cm = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * scale_log2;
                // raise the max used by the exponentials when the true max exceeds it by more than
                // 2^RESCALE_LOG2 (always on the first chunk: m_use = -inf); warp-uniform decision
                const bool raise = c > 0 && !dead && __any_sync(0xffffffffu, cm > m_use + RESCALE_LOG2);
                float alpha = 1.0f;
                if (c == 0) {
                    m_use = cm;
                } else if (raise) {
                    const float m_new = fmaxf(m_use, cm);
                    alpha = ex2f(m_use - m_new);
                    m_use = m_new;
                }
                const float nm = -m_use;
                uint32_t pk[KC / 32][16];
                float csum = 0.0f;
#pragma unroll
                for (int pc = 0; pc < KC / 32; ++pc) {
                    if (!dead && pc < nv) {  // no exponentials for keys past the sequence
#pragma unroll
                        for (int t = 0; t < 32; t += 2) {  // s * scale - max for two keys in one packed FMA
                            float e0, e1;
                            f2_unpack(f2_fma(f2_pack(__uint_as_float(v[pc][t]), __uint_as_float(v[pc][t + 1])),
                                             f2_splat(scale_log2), f2_splat(nm)),
                                      e0, e1);
                            pk[pc][t >> 1] = ex2_h2(e0, e1);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) pk[pc][j] = 0u;
                    }
                    __half2 a[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) a[j] = __hadd2(u32_as_h2(pk[pc][2 * j]), u32_as_h2(pk[pc][2 * j + 1]));
#pragma unroll
                    for (int w = 4; w >= 1; w >>= 1)
#pragma unroll
                        for (int j = 0; j < w; ++j) a[j] = __hadd2(a[j], a[j + w]);
                    csum += __low2float(a[0]) + __high2float(a[0]);
                }
                l_run = l_run * alpha + csum;
                if (g > 0) {
                    // P V of chunk g-1 (this item's or the previous one's) has read P and added to
                    // O: P may be overwritten, O rescaled
                    ok = __all_sync(0xffffffffu, wait_at(B_PVDONE, (g - 1) & 1, CEB_DEVERR_TIMEOUT_EPI));
                    if (!ok) break;
                    tc_fence_after();
                    if (raise) {
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
                if (!dead) {
#pragma unroll
                    for (int pc = 0; pc < KC / 32; ++pc) tmem_st16(row_t + P_COL + (uint32_t)(16 * pc), pk[pc]);
                }
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(B_PFULL));
            }
            // the item's last P V has finished: O / row sum -> fp16 rows of the sequence
            ok = ok && __all_sync(0xffffffffu, wait_at(B_PVDONE, (g - 1) & 1, CEB_DEVERR_TIMEOUT_EPI));
            if (!ok) break;
            if (dead) continue;
            tc_fence_after();
            const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
            uint32_t pk[32];
#pragma unroll
            for (int o0 = 0; o0 < HD; o0 += 32) {
                uint32_t ov[32];
                tmem_ld32(row_t + O_COL + (uint32_t)o0, ov);
                tmem_ld_wait();
#pragma unroll
                for (int t = 0; t < 32; t += 2)
                    pk[(o0 + t) >> 1] =
                        h2_as_u32(__floats2half2_rn(__uint_as_float(ov[t]) * inv, __uint_as_float(ov[t + 1]) * inv));
            }
            const int q = it.q0 + 32 * qd + lane;
            if (q < len) {
                uint4* o = reinterpret_cast<uint4*>(out + (size_t)(it.start + q) * d + it.head * HD);
#pragma unroll
                for (int j = 0; j < 8; ++j) o[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace

// Returns 1 (nothing launched) when the shape is not handled here.
int ceb_attention_fa(const __half* qkv, int total_rows, const int32_t* cu, int n_seqs, int max_len, int d, int n_head,
                     __half* out, int* d_err, cudaStream_t st, int* sched) {
    if (n_head <= 0 || d != n_head * HD || max_len <= 0 || total_rows <= 0 || !sched) return 1;
    if ((reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) return 1;
    if (int rc = ceb_func_smem(reinterpret_cast<const void*>(attn_fa_kernel), SMEM_LAUNCH)) return rc;
    CUtensorMap map;  // Q, K and V tiles: 128 rows x 64 fp16 of the fused qkv rows
    const uint64_t ld_bytes = (uint64_t)3 * d * 2;
    if (int rc = ceb_make_tmap_2d_sw(&map, qkv, 2, (uint64_t)3 * d, (uint64_t)total_rows, ld_bytes, HD, 128, 128))
        return rc;
    const float scale_log2 = (1.0f / sqrtf((float)HD)) * 1.4426950408889634f;
    const int n_qt = (max_len + QT - 1) / QT;
    const int64_t n_items = (int64_t)n_qt * n_head * n_seqs;  // (query tile, head, sequence); empty ones skipped
    if (n_items > INT32_MAX - CTAS_PER_SM * 1024) return 1;     // the counter runs past n_items by one per CTA
    const int grid = (int)std::min<int64_t>(n_items, CTAS_PER_SM * ceb_num_sms());
    CEB_LAUNCH(CEB_PROF_ATTN, st, 0.0, 0.0,
               attn_fa_kernel<<<grid, NTHR, SMEM_LAUNCH, st>>>(map, cu, (int)n_items, n_qt, n_head, d, scale_log2, out,
                                                               d_err, total_rows, max_len, sched));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}
