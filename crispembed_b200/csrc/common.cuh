// common.cuh -- shared device helpers for the sm_100a kernels of crispembed-b200.
//
// Inline-PTX wrappers for mbarriers, TMA (cp.async.bulk.tensor) and the
// tcgen05 tensor-memory / MMA instructions.  Every wait loop here is bounded:
// after CEB_WAIT_LIMIT_CYCLES the wait reports failure, the caller records an
// error code in device memory and unwinds instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define CEB_DEV __device__ __forceinline__

// ~1 s at the B200 boost clock: far above any legitimate wait in these kernels.
#ifndef CEB_WAIT_LIMIT_CYCLES
#define CEB_WAIT_LIMIT_CYCLES 2000000000LL
#endif

// error codes written to the device-side error word
enum ceb_dev_error : int {
    CEB_DEVERR_NONE = 0,
    CEB_DEVERR_TIMEOUT_TMA = 0x101,
    CEB_DEVERR_TIMEOUT_MMA = 0x102,
    CEB_DEVERR_TIMEOUT_DEQ = 0x103,
    CEB_DEVERR_TIMEOUT_EPI = 0x104,
    CEB_DEVERR_BAD_GROUP = 0x105,
    CEB_DEVERR_BAD_INDEX = 0x106,
    CEB_DEVERR_TIMEOUT_PEER = 0x107,  // a peer GPU's signal did not arrive (expert-parallel exchange)
    CEB_DEVERR_EP_OVERFLOW = 0x108,   // expert-parallel rows beyond a receive buffer
};

CEB_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// ------------------------------------------------------------------ system-scope flags (peer GPUs)
CEB_DEV void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
CEB_DEV uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
CEB_DEV uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------------------------------ mbarrier
CEB_DEV void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
CEB_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
CEB_DEV void mbar_arrive(uint32_t bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}
CEB_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
}
CEB_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and raises *abort) on timeout
// or when another role already aborted; the caller must then unwind.
CEB_DEV bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort, int* err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    long long t0 = clock64();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 0) {
            if (abort && *abort) return false;
            if (clock64() - t0 > CEB_WAIT_LIMIT_CYCLES) {
                if (abort) *abort = 1;
                if (err) atomicCAS(err, 0, code);
                return false;
            }
        }
    }
}

// ---------------------------------------------------------------------- TMA
CEB_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            dst),
        "l"(map), "r"(bar), "r"(x), "r"(y)
        : "memory");
}
// contiguous global -> shared bulk copy (16-byte aligned addresses, size a multiple of 16)
CEB_DEV void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// shared -> global tiled store, completion tracked by the issuing thread's bulk groups
CEB_DEV void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map), "r"(src),
                 "r"(x), "r"(y)
                 : "memory");
}
CEB_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until at most N committed bulk groups still read their shared-memory source
template <int N>
CEB_DEV void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
CEB_DEV void bulk_wait() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// make this thread's generic-proxy shared-memory writes visible to the async proxy (TMA, tcgen05)
CEB_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
CEB_DEV void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ------------------------------------------------------------------ tcgen05
// TMEM allocation is warp-wide; the allocated base address is written to smem.
CEB_DEV void tmem_alloc(uint32_t smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_dst), "r"(ncols)
                 : "memory");
}
CEB_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
CEB_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
CEB_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
CEB_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16, fp32 accumulate, 1 CTA.
CEB_DEV void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T
CEB_DEV void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on an mbarrier once every previously issued tcgen05 op of this thread completed.
CEB_DEV void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 32 lanes x 32 bit, 32 consecutive columns: thread t of the warp moves TMEM lane
// (lane_base + t), columns col..col+31.
CEB_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
CEB_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

CEB_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
// 32 lanes x 32 bit, 16 consecutive columns
CEB_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
CEB_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05 format): K-major operand, 128-byte
// swizzle, 8-row core-matrix groups 1024 B apart.  Tile bases must be 1024-B
// aligned; advancing the start address by 32 B steps K by 16 fp16 values.
CEB_DEV uint64_t smem_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFF) >> 4);        // start address  [0,14)
    d |= (uint64_t)1 << 16;                         // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;               // stride byte offset [32,46)
    d |= (uint64_t)1 << 46;                         // descriptor version (sm100)
    d |= (uint64_t)2 << 61;                         // SWIZZLE_128B
    return d;
}

// MN-major operand, 64-byte swizzle: rows of 64 B (32 fp16 along N) consecutive
// along K, 8-row (512 B) swizzle atoms; one atom along N (N <= 32 per CTA).
CEB_DEV uint64_t smem_desc_mn_sw64(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFF) >> 4);        // start address  [0,14)
    d |= (uint64_t)1 << 16;                         // leading byte offset (single atom along N)
    d |= (uint64_t)(512 >> 4) << 32;                // stride byte offset: next 8 K-rows
    d |= (uint64_t)1 << 46;                         // descriptor version (sm100)
    d |= (uint64_t)4 << 61;                         // SWIZZLE_64B
    return d;
}

// Instruction descriptor: kind::f16 with fp16 A/B, fp32 D, both K-major.
CEB_DEV uint32_t idesc_f16_f32(int M, int N) {
    return (1u << 4)                      // D format F32
           | (0u << 7) | (0u << 10)       // A, B = F16
           | ((uint32_t)(N >> 3) << 17)   // N
           | ((uint32_t)(M >> 4) << 24);  // M
}

// ------------------------------------------------- CTA pairs (cluster of 2)
// The pair shares one tcgen05.mma.cta_group::2 (M = 256): each CTA holds half of
// the A rows and half of the B rows in its own shared memory and half of D (its
// 128 lanes x N columns) in its own tensor memory.  Rank 0 issues the MMAs.
CEB_DEV uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// all threads of both CTAs; release/acquire at cluster scope
CEB_DEV void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// address of the same shared-memory location in CTA `rank` of the cluster
CEB_DEV uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
// arrive (release, cluster scope) on an mbarrier given by its cluster address
CEB_DEV void mbar_arrive_cluster(uint32_t cl_bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cl_bar) : "memory");
}
CEB_DEV bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait (acquire at cluster scope) for barriers that other CTAs of the pair arrive on
CEB_DEV bool mbar_wait_cluster(uint32_t bar, uint32_t parity, volatile int* abort, int* err, int code) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    long long t0 = clock64();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((i & 255) == 0) {
            if (abort && *abort) return false;
            if (clock64() - t0 > CEB_WAIT_LIMIT_CYCLES) {
                if (abort) *abort = 1;
                if (err) atomicCAS(err, 0, code);
                return false;
            }
        }
    }
}
CEB_DEV void tmem_alloc_pair(uint32_t smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_dst), "r"(ncols)
                 : "memory");
}
CEB_DEV void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
CEB_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
CEB_DEV void mma_pair_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// A from tensor memory (TS form): each CTA's TMEM holds its M/2 rows of A,
// 32-bit column c = fp16 K elements 2c, 2c+1.
CEB_DEV void mma_pair_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// arrive on the mbarrier at cluster address `cl_bar` when this thread's MMAs complete
CEB_DEV void mma_pair_commit(uint32_t cl_bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cl_bar)
                 : "memory");
}
// shared::cta -> shared::cluster bulk copy (16-byte aligned, size a multiple of 16)
// whose bytes count on the mbarrier at cluster address `cl_bar` (in the
// destination CTA).  Used as an asynchronous, non-blocking cross-CTA signal.
CEB_DEV void bulk_copy_to_cluster(uint32_t cl_dst, uint32_t src, uint32_t bytes, uint32_t cl_bar) {
    asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     cl_dst),
                 "r"(src), "r"(bytes), "r"(cl_bar)
                 : "memory");
}
// 2D tile load into this CTA's shared memory whose completion bytes count on the
// mbarrier at cluster address `cl_bar` (the pair leader's)
CEB_DEV void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t cl_bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
        "%4}], [%2];" ::"r"(dst),
        "l"(map), "r"(cl_bar), "r"(x), "r"(y)
        : "memory");
}

// ------------------------------------------------------------------ numerics
CEB_DEV float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f)); }

CEB_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
CEB_DEV uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
CEB_DEV __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Packed fp32 pairs (sm_100 f32x2 arithmetic): one instruction, two round-to-nearest
// results, each equal to the scalar operation's (no flush to zero, as the scalar code).
struct f32x2 {
    uint64_t v;
};
CEB_DEV f32x2 f2_pack(float lo, float hi) {
    f32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r.v) : "f"(lo), "f"(hi));
    return r;
}
CEB_DEV f32x2 f2_splat(float a) { return f2_pack(a, a); }
CEB_DEV void f2_unpack(f32x2 a, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(a.v)); }
CEB_DEV f32x2 f2_fma(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d.v) : "l"(a.v), "l"(b.v), "l"(c.v));
    return d;
}
CEB_DEV f32x2 f2_mul(f32x2 a, f32x2 b) {
    f32x2 d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d.v) : "l"(a.v), "l"(b.v));
    return d;
}
CEB_DEV f32x2 f2_add(f32x2 a, f32x2 b) {
    f32x2 d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d.v) : "l"(a.v), "l"(b.v));
    return d;
}

// Four int8 values -> two half2 holding d*q (each product rounded once to fp16).
// q+128 is placed in the low mantissa byte of fp16 1024 (0x64xx), then 1152 is
// subtracted exactly, leaving q as an fp16 integer.
CEB_DEV void i8x4_to_h2x2(uint32_t w, __half2 d2, uint32_t& lo, uint32_t& hi) {
    const uint32_t t = w ^ 0x80808080u;
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
    __half2 a = __hsub2(u32_as_h2(prmt(t, 0x64646464u, 0x4140u)), bias);
    __half2 b = __hsub2(u32_as_h2(prmt(t, 0x64646464u, 0x4342u)), bias);
    lo = h2_as_u32(__hmul2(a, d2));
    hi = h2_as_u32(__hmul2(b, d2));
}

#define CEB_CUDA_OK(expr)                                     \
    do {                                                      \
        cudaError_t e__ = (expr);                             \
        if (e__ != cudaSuccess) return ceb_set_cuda_error(e__, #expr, __FILE__, __LINE__); \
    } while (0)

// ------------------------------------------------------------------ exp2 on the FMA pipe
// 2^x for x <= 0 on the FMA pipe, so attention softmaxes can share their
// exponentials between the MUFU unit and the FMA pipe.  x = n + f with
// n = rint(x) (the 1.5*2^23 rounding constant) and f in [-0.5, 0.5]; 2^f by a
// degree-4 polynomial fitted here for relative error on [-0.5, 0.5] (weighted
// least squares, Lawson iterations: max relative error 2.7e-6 in fp32, far below
// the fp16 rounding of P); 2^n enters through the exponent field.  x is clamped
// at -125 so the result stays a normal float (2^-125 rounds to 0 in fp16 P).
CEB_DEV float ex2_poly(float x) {
    x = fmaxf(x, -125.0f);
    const float t = x + 12582912.0f;
    const float n = t - 12582912.0f;
    const float f = x - n;
    float p = 0.009570101276040077f;
    p = fmaf(p, f, 0.05591785907745361f);
    p = fmaf(p, f, 0.240247443318367f);
    p = fmaf(p, f, 0.6931217908859253f);
    p = fmaf(p, f, 0.9999992847442627f);
    const uint32_t e = (uint32_t)(__float_as_int(t) - 0x4B400000) << 23;  // n in the exponent field
    return __uint_as_float(__float_as_uint(p) + e);
}
