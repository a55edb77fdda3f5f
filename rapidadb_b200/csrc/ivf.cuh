// Probe inversion shared by the IVF list scans (internal interface): the
// Q x nprobe (query, probed list) entries of a search, grouped by list.
#pragma once

#include "common.cuh"

namespace rdb {

struct IvfWs {
    size_t off_lab, off_perm, off_seg, off_qv, off_sort, bytes;
};

// Workspace layout of the inversion: list labels of the entries, the
// entries sorted by list (perm: entry e = query * nprobe + slot), segment
// starts [nlist + 1], per-query values [Q], sort scratch.
IvfWs ivf_ws(int64_t Q, int nprobe, int nlist);
// perm / seg of w from probe [Q, nprobe] (stable: entries of a list in
// ascending entry order)
int invert_probes(const int64_t* probe, int64_t Q, int nprobe, int nlist, const IvfWs& w, char* base,
                  cudaStream_t s);

}  // namespace rdb
