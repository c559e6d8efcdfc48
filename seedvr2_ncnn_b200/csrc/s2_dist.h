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
    int wait_ready();
    int fail(int code);
    int all_reduce_sum_f32(float* buf, size_t count, cudaStream_t stream);
    int exchange_bf16(const void* send, const std::vector<int>& send_counts, const std::vector<int>& send_off,
                      void* recv, const std::vector<int>& recv_counts, const std::vector<int>& recv_off,
                      size_t row_elems, cudaStream_t stream);
    int sync(cudaStream_t stream);
};

// Row gather / scatter of bf16 rows (row_elems multiple of 8):
//   gather:  dst[i] = src[idx[i]]     scatter: dst[idx[i]] = src[i]
int launch_gather_rows_bf16(Context& ctx, const void* src, const int* idx, int count, int row_elems, void* dst);
int launch_scatter_rows_bf16(Context& ctx, const void* src, const int* idx, int count, int row_elems, void* dst);

} // namespace s2
