// Stable counting sort of ids by a small integer label (internal interface).
#pragma once

#include "common.cuh"

namespace rdb {

constexpr int kMaxLabels = 16384;  // shared-memory histogram / cursor limit

size_t label_sort_workspace(int64_t n, int K);
// Loads this file's kernels into the current context (CUDA loads them lazily).
int label_sort_preload();

// perm[seg_start[c] .. seg_start[c + 1]) = the ids i with labels[i] == c, in
// ascending i (stable); counts[c] = segment sizes (counts may be NULL).
int label_sort(const int32_t* labels, int64_t n, int K, int64_t* seg_start, int64_t* perm, int64_t* counts,
               void* ws, size_t ws_bytes, cudaStream_t s);

}  // namespace rdb
