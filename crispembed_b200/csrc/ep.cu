// ep.cu -- expert parallelism of the MoE blocks across the GPUs of one node.
//
// The reference runs every expert of a block on one device inside
// ggml_mul_mat_id (src/crispembed.cpp:1365-1371).  Here rank r of `world`
// processes (one per GPU) owns experts [r*E_loc, (r+1)*E_loc) and routes its own
// tokens (data-parallel sequence shards above the experts).  Per MoE block:
//
//   scan_kernel     local expert totals -> row r of every rank's count matrix,
//                   then a release of each rank's counts flag   (moe.cu)
//   ep_wait         counts of every rank present                (bounded)
//   scatter_kernel  each (token, slot) row stored straight into the receive
//                   buffer of its expert's owner over NVLink, last CTA releases
//                   the dispatch flags                          (moe.cu)
//   ep_wait         every rank's rows for the local experts present
//   fc1+GELU, fc2   grouped tcgen05 GEMMs over the local experts' rows
//   ep_return       each output row stored back into its source rank's ret
//                   buffer at the source's own permutation position, last CTA
//                   releases the return flags
//   ep_wait         every local (token, slot) output present; the combine then
//                   runs exactly as on one GPU.
//
// No host synchronisation, no collective library call: the exchange is done by
// the kernels that produce the data, with plain peer stores.
// Every row keeps its K-loop order, so results are bit-identical to one GPU.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "ceb_encoder_internal.h"
#include "ceb_ep_internal.h"
#include "ceb_internal.h"
#include "common.cuh"
#include "../../include/ceb_ops.h"

namespace {

constexpr uint64_t EP_MAGIC = 0x3142504542454320ull;  // region header tag
constexpr int EP_MAXE = 64;

__global__ void ep_wait_kernel(const uint32_t* __restrict__ flags, int world, uint32_t epoch, uint64_t timeout_ns,
                               int* err) {
    const int p = threadIdx.x;
    if (p < world) {
        const uint64_t t0 = global_timer_ns();
        uint32_t it = 0;
        while ((int)(ld_acquire_sys(flags + p) - epoch) < 0) {
            if ((++it & 31) == 0 && global_timer_ns() - t0 > timeout_ns) {
                atomicCAS(err, 0, (int)CEB_DEVERR_TIMEOUT_PEER | (p << 12));
                break;
            }
            __nanosleep(200);
        }
    }
    __syncthreads();
}

// Output rows of the local experts back to their source ranks.  The receive
// order is segments (local expert el, source p) in increasing start; segment
// (el, p) goes to p's ret rows from p's own offset of expert r*E_loc+el.
__global__ void __launch_bounds__(256)
    ep_return_kernel(const __half* __restrict__ down, int d, int E, ceb_ep_args ep, int* err) {
    __shared__ int seg_start[EP_MAXE + 1];
    __shared__ long long seg_dst[EP_MAXE];
    __shared__ int seg_peer[EP_MAXE];
    const int nseg = ep.E_loc * ep.world;
    if (threadIdx.x < nseg) {
        const int s = threadIdx.x, el = s / ep.world, p = s - el * ep.world, g = ep.rank * ep.E_loc + el;
        int start = ep.offsets_recv[el];
        for (int p2 = 0; p2 < p; ++p2) start += ep.C[p2 * E + g];
        long long dst = 0;
        for (int g2 = 0; g2 < g; ++g2) dst += ep.C[p * E + g2];
        seg_start[s] = start;
        seg_dst[s] = dst;
        seg_peer[s] = p;
    }
    if (threadIdx.x == 0) seg_start[nseg] = ep.offsets_recv[ep.E_loc];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
    const int total = seg_start[nseg];
    for (int r = blockIdx.x * wpb + warp; r < total; r += gridDim.x * wpb) {
        int s = 0;
        while (s + 1 < nseg && seg_start[s + 1] <= r) ++s;
        const long long row = seg_dst[s] + (r - seg_start[s]);
        if (row < 0 || row >= ep.ret_rows) {
            if (lane == 0) atomicCAS(err, 0, (int)CEB_DEVERR_EP_OVERFLOW);
            continue;
        }
        // fp16 rows: 16 bytes (8 values) per lane and step, d / 256 steps
        const uint4* src = reinterpret_cast<const uint4*>(down + (size_t)r * d);
        uint4* dst = reinterpret_cast<uint4*>(ep.peers[seg_peer[s]].ret + (size_t)row * d);
        const int nu = d / 8;  // uint4 per row
        uint4 v[4];            // the whole row in flight before the peer stores (d <= 1024)
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (i * 32 + lane < nu) v[i] = __ldg(src + i * 32 + lane);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (i * 32 + lane < nu) dst[i * 32 + lane] = v[i];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        if (atomicAdd(ep.done + 1, 1) == (int)gridDim.x - 1) {
            atomicExch(ep.done + 1, 0);
            __threadfence_system();
            for (int p = 0; p < ep.world; ++p)
                st_release_sys(ep.peers[p].flags + CEB_EPF_RETURN * ep.world + ep.rank, ep.epoch);
        }
    }
}

size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

struct RegionLayout {
    size_t o_recv, o_ret, o_counts, o_flags, bytes;
};

RegionLayout region_layout(int world, int E, int K, int d, int T_cap, int64_t recv_rows) {
    RegionLayout L;
    size_t off = align256(sizeof(ceb_ep_header));
    L.o_recv = off;
    off += align256((size_t)recv_rows * d * 2);
    L.o_ret = off;
    off += align256((size_t)T_cap * K * d * 2);
    L.o_counts = off;
    off += align256((size_t)2 * world * E * 4);
    L.o_flags = off;
    off += align256((size_t)CEB_EPF_ROWS * world * 4);
    L.bytes = off;
    return L;
}

ceb_ep_peer peer_at(uint8_t* base, const RegionLayout& L) {
    ceb_ep_peer p;
    p.recv = reinterpret_cast<__half*>(base + L.o_recv);
    p.ret = reinterpret_cast<__half*>(base + L.o_ret);
    p.counts = reinterpret_cast<int32_t*>(base + L.o_counts);
    p.flags = reinterpret_cast<uint32_t*>(base + L.o_flags);
    return p;
}

void ep_release(ceb_ep* ep) {
    if (!ep) return;
    cudaSetDevice(ep->device);
    for (void* p : ep->opened)
        if (p) cudaIpcCloseMemHandle(p);
    ep->opened.clear();
    for (void* p : {(void*)ep->region, (void*)ep->d_peers, (void*)ep->h, (void*)ep->down, (void*)ep->offsets_recv,
                    (void*)ep->done})
        if (p) cudaFree(p);
    ep->region = nullptr;
}

int ep_upload_peers(ceb_ep* ep, const std::vector<ceb_ep_peer>& peers) {
    CEB_CUDA_OK(cudaMemcpy(ep->d_peers, peers.data(), peers.size() * sizeof(ceb_ep_peer), cudaMemcpyHostToDevice));
    return 0;
}

}  // namespace

ceb_wplane ceb_wplane_slice(const ceb_wplane& w, int g0, int n) {
    ceb_wplane s = w;
    const size_t per_q = w.n_groups ? w.q_bytes / w.n_groups : 0;
    const size_t per_s = w.n_groups ? w.s_bytes / w.n_groups : 0;
    s.n_groups = n;
    s.q = w.q + per_q * g0;
    s.q_bytes = per_q * n;
    s.s_bytes = per_s * n;
    return s;
}

int ceb_ep_wait(const ceb_ep_args& a, int row, int* dev_err, cudaStream_t st) {
    CEB_LAUNCH(CEB_PROF_EP_WAIT, st, 0.0, 0.0,
               ep_wait_kernel<<<1, 32, 0, st>>>(a.my_flags + (size_t)row * a.world, a.world, a.epoch, a.timeout_ns,
                                                dev_err));
    CEB_CUDA_OK(cudaGetLastError());
    return 0;
}

int ceb_ep_moe(ceb_ep* ep, const ceb_moe_weights& mwl, const void* x, int x_dtype, const __half* x16, int T,
               const ceb_moe_ws& ws, int* dev_err, cudaStream_t st) {
    if (!ep || !ep->connected) return ceb_set_error(1, "expert parallel: not connected");
    if (T < 0 || T > ep->T_cap)
        return ceb_set_error(1, "expert parallel: %d local tokens exceed the capacity of %d", T, ep->T_cap);
    if (mwl.n_experts != ep->E || mwl.top_k != ep->K || mwl.d != ep->d || mwl.ffn != ep->F ||
        mwl.fc1.n_groups != ep->E_loc || mwl.fc2.n_groups != ep->E_loc)
        return ceb_set_error(1, "expert parallel: block shape (E=%d K=%d d=%d F=%d, %d local experts) does not match "
                                "the exchange (E=%d K=%d d=%d F=%d, %d local)",
                             mwl.n_experts, mwl.top_k, mwl.d, mwl.ffn, mwl.fc1.n_groups, ep->E, ep->K, ep->d, ep->F,
                             ep->E_loc);
    const uint32_t epoch = ++ep->epoch;
    ceb_ep_args a;
    a.peers = ep->d_peers;
    a.par = (int)(epoch & 1u);
    a.C = ep->self.counts + (size_t)a.par * ep->world * ep->E;
    a.my_offsets = ws.offsets;
    a.offsets_recv = ep->offsets_recv;
    a.done = ep->done;
    a.my_flags = ep->self.flags;
    a.rank = ep->rank;
    a.world = ep->world;
    a.E_loc = ep->E_loc;
    a.recv_rows = ep->recv_rows;
    a.ret_rows = (int64_t)ep->T_cap * ep->K;
    a.timeout_ns = (uint64_t)ep->timeout_ms * 1000000ull;
    a.epoch = epoch;
    int rc = ceb_moe_permute(mwl, x, x_dtype, x16, T, ws, nullptr, &a, dev_err, st);
    if (rc) return rc;
    if ((rc = ceb_ep_wait(a, CEB_EPF_DISPATCH, dev_err, st))) return rc;
    const int rows = (int)ep->recv_rows;
    ceb_gemm_args a1;
    a1.offsets = ep->offsets_recv;
    a1.m_rows = rows;
    a1.out = ep->h;
    a1.ldo = ep->F;
    a1.epi = CEB_EPI_F16_OUT | CEB_EPI_GELU;
    a1.err = dev_err;
    a1.prof_cat = CEB_PROF_MOE_GEMM;
    if ((rc = ceb_gemm_launch(mwl.fc1, ep->self.recv, rows, a1, st))) return rc;
    ceb_gemm_args a2;
    a2.offsets = ep->offsets_recv;
    a2.m_rows = rows;
    a2.out = ep->down;
    a2.ldo = ep->d;
    a2.epi = CEB_EPI_F16_OUT;
    a2.err = dev_err;
    a2.prof_cat = CEB_PROF_MOE_GEMM;
    if ((rc = ceb_gemm_launch(mwl.fc2, ep->h, rows, a2, st))) return rc;
    const int grid = 2 * ceb_num_sms();
    CEB_LAUNCH(CEB_PROF_EXCHANGE, st, 0.0, 0.0,
               ep_return_kernel<<<grid, 256, 0, st>>>(ep->down, ep->d, ep->E, a, dev_err));
    CEB_CUDA_OK(cudaGetLastError());
    return ceb_ep_wait(a, CEB_EPF_RETURN, dev_err, st);
}

// ------------------------------------------------------------------ C ABI

extern "C" ceb_ep* ceb_ep_create(int rank, int world, int n_experts, int top_k, int d, int ffn,
                                 int max_local_tokens) {
    if (world < 1 || world > 32 || rank < 0 || rank >= world || n_experts < 1 || n_experts > 32 ||
        n_experts % world || top_k < 1 || top_k > n_experts || top_k > 4 || d <= 0 || d % 128 || d > 1024 ||
        ffn <= 0 || ffn % 128 || max_local_tokens < 1) {
        ceb_set_error(1, "ep_create: unsupported arguments (rank %d of %d, E=%d, K=%d, d=%d, F=%d, T=%d)", rank,
                      world, n_experts, top_k, d, ffn, max_local_tokens);
        return nullptr;
    }
    ceb_ep* ep = new ceb_ep();
    ep->rank = rank;
    ep->world = world;
    ep->E = n_experts;
    ep->E_loc = n_experts / world;
    ep->K = top_k;
    ep->d = d;
    ep->F = ffn;
    ep->T_cap = max_local_tokens;
    // worst case: every (token, slot) of every rank that can land on this rank's experts
    ep->recv_rows = (int64_t)world * max_local_tokens * std::min(top_k, ep->E_loc);
    if (ep->recv_rows > (int64_t)1 << 30) {
        ceb_set_error(1, "ep_create: receive capacity of %lld rows is too large", (long long)ep->recv_rows);
        delete ep;
        return nullptr;
    }
    cudaGetDevice(&ep->device);
    const RegionLayout L = region_layout(world, n_experts, top_k, d, max_local_tokens, ep->recv_rows);
    ep->region_bytes = L.bytes;
    bool ok = cudaMalloc(&ep->region, L.bytes) == cudaSuccess &&
              cudaMalloc(&ep->h, (size_t)ep->recv_rows * ffn * 2) == cudaSuccess &&
              cudaMalloc(&ep->down, (size_t)ep->recv_rows * d * 2) == cudaSuccess &&
              cudaMalloc(&ep->offsets_recv, (size_t)(ep->E_loc + 1) * 4) == cudaSuccess &&
              cudaMalloc(&ep->done, 4 * sizeof(int)) == cudaSuccess &&
              cudaMalloc(&ep->d_peers, (size_t)world * sizeof(ceb_ep_peer)) == cudaSuccess;
    if (ok) {
        ceb_ep_header h{};
        h.magic = EP_MAGIC;
        h.world = world;
        h.n_experts = n_experts;
        h.top_k = top_k;
        h.d = d;
        h.ffn = ffn;
        h.t_cap = max_local_tokens;
        h.recv_rows = ep->recv_rows;
        uint8_t* base = static_cast<uint8_t*>(ep->region);
        ok = cudaMemcpy(base, &h, sizeof(h), cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemset(base + L.o_counts, 0, L.bytes - L.o_counts) == cudaSuccess &&
             cudaMemset(ep->offsets_recv, 0, (size_t)(ep->E_loc + 1) * 4) == cudaSuccess &&
             cudaMemset(ep->done, 0, 4 * sizeof(int)) == cudaSuccess;
        ep->self = peer_at(base, L);
    }
    if (!ok) {
        ceb_set_error(4, "ep_create: out of device memory (%.2f GB region)", L.bytes / 1e9);
        ep_release(ep);
        delete ep;
        return nullptr;
    }
    if (world == 1) {
        ep->opened.assign(1, nullptr);
        if (ep_upload_peers(ep, {ep->self})) {
            ep_release(ep);
            delete ep;
            return nullptr;
        }
        ep->connected = true;
    }
    return ep;
}

extern "C" int ceb_ep_ipc_handle(const ceb_ep* ep, void* handle_out) {
    if (!ep || !handle_out) return ceb_set_error(1, "ep_ipc_handle: bad arguments");
    static_assert(sizeof(cudaIpcMemHandle_t) == CEB_EP_HANDLE_BYTES, "IPC handle size");
    cudaIpcMemHandle_t h;
    CEB_CUDA_OK(cudaIpcGetMemHandle(&h, ep->region));
    memcpy(handle_out, &h, sizeof(h));
    return 0;
}

extern "C" int ceb_ep_connect(ceb_ep* ep, const void* handles) {
    if (!ep || !handles) return ceb_set_error(1, "ep_connect: bad arguments");
    if (ep->connected) return 0;
    const RegionLayout L = region_layout(ep->world, ep->E, ep->K, ep->d, ep->T_cap, ep->recv_rows);
    std::vector<ceb_ep_peer> peers(ep->world);
    ep->opened.assign(ep->world, nullptr);
    const uint8_t* hb = static_cast<const uint8_t*>(handles);
    for (int p = 0; p < ep->world; ++p) {
        if (p == ep->rank) {
            peers[p] = ep->self;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, hb + (size_t)p * CEB_EP_HANDLE_BYTES, sizeof(h));
        void* base = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return ceb_set_cuda_error(e, "IPC open of a peer's exchange region", __FILE__, __LINE__);
        ep->opened[p] = base;
        ceb_ep_header hp{};
        CEB_CUDA_OK(cudaMemcpy(&hp, base, sizeof(hp), cudaMemcpyDefault));
        if (hp.magic != EP_MAGIC || hp.world != ep->world || hp.n_experts != ep->E || hp.top_k != ep->K ||
            hp.d != ep->d || hp.ffn != ep->F || hp.t_cap != ep->T_cap || hp.recv_rows != ep->recv_rows)
            return ceb_set_error(1, "ep_connect: rank %d's exchange region has a different shape", p);
        peers[p] = peer_at(static_cast<uint8_t*>(base), L);
    }
    if (int rc = ep_upload_peers(ep, peers)) return rc;
    ep->connected = true;
    return 0;
}

extern "C" void ceb_ep_set_timeout_ms(ceb_ep* ep, int ms) {
    if (ep && ms > 0) ep->timeout_ms = ms;
}

extern "C" void ceb_ep_free(ceb_ep* ep) {
    if (!ep) return;
    cudaDeviceSynchronize();
    ep_release(ep);
    delete ep;
}

extern "C" int ceb_moe_ffn_ep(const ceb_moe_layer* L, ceb_ep* ep, const void* d_x, int x_dtype, int n_tokens,
                              float* d_y, void* d_workspace, size_t workspace_bytes, void* stream) {
    if (!L || !ep || n_tokens < 0 || !d_workspace || (n_tokens > 0 && (!d_x || !d_y)))
        return ceb_set_error(1, "moe_ffn_ep: bad arguments");
    if (x_dtype != CEB_ACT_F32 && x_dtype != CEB_ACT_BF16 && x_dtype != CEB_ACT_F16)
        return ceb_set_error(1, "moe_ffn_ep: x_dtype %d unsupported", x_dtype);
    const size_t need = ceb_moe_workspace_size(L, std::max(n_tokens, 1));
    if (workspace_bytes < need)
        return ceb_set_error(1, "moe_ffn_ep: workspace of %zu bytes, %zu needed", workspace_bytes, need);
    if (reinterpret_cast<uintptr_t>(d_workspace) & 255) return ceb_set_error(1, "moe_ffn_ep: workspace not 256-B aligned");
    const ceb_moe_weights& w = L->w;
    if (w.n_experts != ep->E) return ceb_set_error(1, "moe_ffn_ep: layer has %d experts, exchange %d", w.n_experts, ep->E);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    ceb_moe_ws ws;
    ceb_moe_ws_layout(std::max(n_tokens, 1), w.d, w.n_experts, w.top_k, w.ffn, &ws, static_cast<uint8_t*>(d_workspace));
    int* err = ceb_op_error_word();
    if (!err) return ceb_set_error(4, "out of device memory");
    int rc = ceb_moe_route(w, d_x, x_dtype, n_tokens, ws, nullptr, st);
    if (rc) return rc;
    ceb_moe_weights wl = w;
    wl.fc1 = ceb_wplane_slice(w.fc1, ep->rank * ep->E_loc, ep->E_loc);
    wl.fc2 = ceb_wplane_slice(w.fc2, ep->rank * ep->E_loc, ep->E_loc);
    if ((rc = ceb_ep_moe(ep, wl, d_x, x_dtype, nullptr, n_tokens, ws, err, st))) return rc;
    return ceb_moe_combine(ep->self.ret, ws.slot_pos, ws.wts, n_tokens, w.d, w.top_k, w.bias, d_y, st);
}
