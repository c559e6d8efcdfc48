// Multi-GPU declarations: token-ownership plan and the NCCL communicator.
#pragma once

#include <nccl.h>

#include <vector>

#include "s2_internal.h"

namespace s2 {

// Token ownership of one sample for `world` ranks, seen from `rank`.
// Per window plan p (0 = unshifted, 1 = shifted): each window has one owner
// (the rank holding most of its tokens); foreign rows of its tokens travel to
// it before attention and their context rows travel back.
struct ShardPlan
{
    int world = 1, rank = 0, Nv = 0, T = 0;
    Plan plan[2];                          // unshifted / shifted window plans
    std::vector<int> token_owner;          // [Nv] owning rank of each video token
    std::vector<int> token_local;          // [Nv] row of the token at its owner
    std::vector<int> n_local;              // [world] owned video tokens per rank
    std::vector<int> local_tokens;         // this rank's tokens (global ids) in row order
    std::vector<int> owner[2];             // window -> rank
    std::vector<int> win_mine[2];          // this rank's windows
    // Rows of this rank's buffers for each global token: own rows first,
    // then (after the text rows) the foreign rows received; -1 elsewhere.
    std::vector<int> row[2];
    std::vector<std::vector<int>> send_rows[2];   // [world] own rows sent to each rank (its order)
    std::vector<std::vector<int>> send_tokens[2]; // [world] the same rows as global token ids
    std::vector<std::vector<int>> recv_tokens[2]; // [world] foreign tokens received from each rank
    std::vector<int> send_off[2], recv_off[2];    // [world] prefix offsets (rows)
    int m_foreign[2] = {0, 0}, m_send[2] = {0, 0};
    // every rank's view: recv_off_all[p][q * world + s] = where rank q stores
    // the rows it receives from rank s (after its own rows and text rows);
    // m_foreign_all[p][q] = rows rank q receives
    std::vector<int> recv_off_all[2], m_foreign_all[2];
};

int build_shard(const int* shape, int text_length, const int* window, int window_mode, int rank, int world,
                ShardPlan& sp);

bool nccl_available();
int nccl_unique_id(void* out128);

struct Dist
{
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    int timeout_ms = 60000;
    bool aborted = false;
    int init(const void* id128, int rank, int world, int timeout_ms);
    void destroy();
    int wait_ready(Context* ctx = nullptr);
    int fail(int code);
    int all_reduce_sum_f32(Context& ctx, float* buf, size_t count);
    int exchange_bf16(Context& ctx, const void* send, const std::vector<int>& send_counts,
                      const std::vector<int>& send_off, void* recv, const std::vector<int>& recv_counts,
                      const std::vector<int>& recv_off, size_t row_elems);
    int sync(cudaStream_t stream);
    // Maps every rank's `local` allocation into this process (CUDA IPC, handles
    // all-gathered over NCCL); peers[r] is rank r's base (peers[rank] = local).
    int share_buffer(Context& ctx, void* local, std::vector<void*>& peers);
    std::vector<void*> opened; // IPC mappings to close on destroy
    uint32_t epoch = 0;        // cross-GPU barrier generation
};

// NVLink peer-memory kernels (peer.cu)
int launch_push_rows(Context& ctx, const void* src, int row_elems, const int4* table, int count, void* const* dst,
                     int world);
int launch_peer_barrier(Context& ctx, void* const* peer_flags, uint32_t* my_flags, int rank, int world,
                        uint32_t epoch);
int launch_text_reduce_peers(Context& ctx, void* const* parts, int world, int64_t count, void* out_bf16);

// Row gather / scatter of bf16 rows (row_elems multiple of 8):
//   gather:  dst[i] = src[idx[i]]     scatter: dst[idx[i]] = src[i]
int launch_gather_rows_bf16(Context& ctx, const void* src, const int* idx, int count, int row_elems, void* dst);
int launch_scatter_rows_bf16(Context& ctx, const void* src, const int* idx, int count, int row_elems, void* dst);

} // namespace s2
