// Paged KV cache addressing shared by the host code and the kernels.
#pragma once

namespace cb {

// The cache of a layer is a pool of pages of 2^shift token rows; logical row c of sequence b
// lives in physical row (table[b * pps + (c >> shift)] << shift) + (c & (2^shift - 1)).
// table == nullptr is the contiguous layout (the degenerate case: sequence b's rows at b's
// per-sequence stride), which the raw C-ABI attention entry points always use.
struct KvPaging {
    const int* table = nullptr;  // [sequences, pps] physical page ids
    int shift = 0;
    int pps = 0;                 // table entries per sequence
};

}  // namespace cb
