// ceb_ep_internal.h -- expert parallelism across the GPUs of one node.
//
// One process per GPU; rank r owns experts [r*E_loc, (r+1)*E_loc) of every MoE
// block and routes its own tokens.  Every rank exports one device region through
// CUDA IPC and maps the regions of its peers, so the exchange steps are plain
// stores into peer memory over NVLink, issued by the kernels that produce the
// data; completion travels as release/acquire flags tagged with a per-block
// epoch, and every wait is bounded (CEB_DEVERR_TIMEOUT_PEER on expiry).
//
// Region of rank r (identical layout on every rank):
//   header  : ceb_ep_header (shape check at connect time)
//   recv    : [recv_rows x d] fp16  rows of r's experts, expert-major, then by
//             source rank, then in the source's stable (token, slot) order
//   ret     : [T_cap*K x d] fp16    expert outputs of r's own (token, slot)s,
//             in r's local expert-major order (the single-GPU permutation)
//   counts  : [2][world][E] int32   per-source expert counts (epoch parity)
//   flags   : [3][world] uint32     counts / dispatch / return done, by source
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include <vector>

#include "ceb_moe_internal.h"

struct ceb_ep_peer {
    __half* recv;
    __half* ret;
    int32_t* counts;
    uint32_t* flags;
};

enum { CEB_EPF_COUNTS = 0, CEB_EPF_DISPATCH = 1, CEB_EPF_RETURN = 2, CEB_EPF_ROWS = 3 };

struct ceb_ep_header {
    uint64_t magic;
    int32_t world, n_experts, top_k, d, ffn, t_cap;
    int64_t recv_rows;
};

struct ceb_ep {
    int rank = 0, world = 1, E = 0, E_loc = 0, K = 0, d = 0, F = 0, T_cap = 0;
    int64_t recv_rows = 0;
    int device = 0;
    int timeout_ms = 2000;
    uint32_t epoch = 0;
    bool connected = false;
    void* region = nullptr;
    size_t region_bytes = 0;
    ceb_ep_peer self{};
    std::vector<void*> opened;        // peer regions mapped through IPC (nullptr for self)
    ceb_ep_peer* d_peers = nullptr;   // device [world]
    // local (not exported) buffers
    __half* h = nullptr;              // [recv_rows x F] fc1 output
    __half* down = nullptr;           // [recv_rows x d] fc2 output
    int32_t* offsets_recv = nullptr;  // [E_loc + 1] row ranges of the local experts in recv
    int* done = nullptr;              // [2] completion counters of the dispatch / return kernels
};

// Kernel-side view of one exchange (passed by value).
struct ceb_ep_args {
    const ceb_ep_peer* peers = nullptr;  // null: single-GPU path
    const int32_t* C = nullptr;          // this epoch's count matrix [world][E] in the local region
    const int32_t* my_offsets = nullptr; // [E+1] local expert-major offsets (single-GPU permutation)
    int32_t* offsets_recv = nullptr;
    int* done = nullptr;                 // [2] completion counters (dispatch, return)
    const uint32_t* my_flags = nullptr;  // [CEB_EPF_ROWS][world] flags in the local region
    int rank = 0, world = 1, E_loc = 0, par = 0;
    int64_t recv_rows = 0, ret_rows = 0;
    uint64_t timeout_ns = 0;
    uint32_t epoch = 0;
};

// Bounded wait (one launch, one thread per source rank) until every rank's flag
// of the given row reaches a.epoch; CEB_DEVERR_TIMEOUT_PEER on expiry.
int ceb_ep_wait(const ceb_ep_args& a, int row, int* dev_err, cudaStream_t st);

// The MoE block's exchange + expert products on rank ep->rank.  Routes must be in
// ws (ids, wts, block_counts) for the T local tokens; x16 (or x) holds their rows.
// mw_local: fc1/fc2 planes holding the E_loc local experts (router unused here).
// On return (stream order) ep->self.ret holds the expert outputs of the local
// (token, slot)s at ws.slot_pos, ready for the combine.
int ceb_ep_moe(ceb_ep* ep, const ceb_moe_weights& mw_local, const void* x, int x_dtype, const __half* x16, int T,
               const ceb_moe_ws& ws, int* dev_err, cudaStream_t st);

// Expert-slice view of a grouped weight plane (no copy).
ceb_wplane ceb_wplane_slice(const ceb_wplane& w, int g0, int n);

// moe.cu pieces the exchange is built from
int ceb_moe_route(const ceb_moe_weights& mw, const void* x, int x_dtype, int T, const ceb_moe_ws& ws,
                  float* logits_out, cudaStream_t st);
// scan (+ count publication) -> [wait for every rank's counts] -> scatter (+ dispatch)
int ceb_moe_permute(const ceb_moe_weights& mw, const void* x, int x_dtype, const __half* x16, int T,
                    const ceb_moe_ws& ws, int32_t* expert_counts, const ceb_ep_args* ep, int* dev_err,
                    cudaStream_t st);
int ceb_moe_combine(const __half* down, const int32_t* slot_pos, const float* wts, int T, int d, int K,
                    const float* bias, float* y, cudaStream_t st);
