// Internal helpers shared by the host (.cpp) and device (.cu) parts of libs2b200.
#pragma once

#include <cstdarg>
#include <cstdio>
#include <string>
#include <vector>

#include "s2_b200.h"

namespace s2 {

// Thread-local last error (s2_last_error); set_error returns `st` for
// `return set_error(...)` chains.
s2_status set_error(s2_status st, const char *fmt, ...);
void clear_error();

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// The sharded step's window ownership (s2_shard_windows_joint) of both window
// kinds and rank `rank`'s view of it: the windows it owns (ids), its local token
// order (tok: patched-grid token per local row), and the row exchange from kind
// k to kind 1 - k -- src[k]: local rows of kind k to send, destination rank by
// destination rank (send_count), each in the destination's local order of kind
// 1 - k; dst[k]: where the received rows go in this rank's local order of kind
// 1 - k, source rank by source rank (recv_count). moved_rows[k]: tokens whose
// owner changes from kind k to kind 1 - k (all ranks). dest_rank[k][i] /
// dest_row[k][i]: the rank that holds this rank's kind-k local row i under
// kind 1 - k, and the row's index in that rank's kind-(1 - k) local order.
struct ShardMaps {
    std::vector<int32_t> ids[2], tok[2], src[2], dst[2], dest_rank[2], dest_row[2];
    std::vector<int32_t> send_count[2], recv_count[2];
    long long moved_rows[2] = {0, 0};
};
s2_status shard_exchange_maps(int T, int H, int W, int wt, int wh, int ww, int text_len, int n_ranks, int rank,
                              ShardMaps &maps);

// Failure injection for tests (s2_debug_attention_fault): hands the next
// s2_window_attention launch its K tile to leave out (-1: none) and its wait
// limit, then resets both (one shot).
void take_attention_fault(int *skip_k, unsigned long long *wait_ns);

// Attention core tiling shared by the planner and the kernel.
constexpr int kTileM = 128;   // query rows per Q tile (one TMEM lane per row)
constexpr int kQTiles = 2;    // Q tiles per CTA (one softmax warpgroup each)
constexpr int kCtaRows = kTileM * kQTiles;
constexpr int kTileN = 128;   // key/value rows per pipeline stage

}  // namespace s2
