// Internal helpers shared by the host (.cpp) and device (.cu) parts of libs2b200.
#pragma once

#include <cstdarg>
#include <cstdio>
#include <string>

#include "s2_b200.h"

namespace s2 {

// Thread-local last error (s2_last_error); set_error returns `st` for
// `return set_error(...)` chains.
s2_status set_error(s2_status st, const char *fmt, ...);
void clear_error();

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

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
