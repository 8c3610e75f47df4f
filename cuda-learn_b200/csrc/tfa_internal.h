// Host-side helpers shared between the C-ABI translation units.
#pragma once

#include <cstddef>

#include "../../include/tfa.h"

namespace tfa {

// The forward used by tfa_fwd / tfa_fwd_timed: validation, split-KV plan, TMA
// descriptors and launches on `stream`, with the caller's workspace. ev_begin / ev_end
// (cudaEvent_t or NULL) are recorded around the attention kernel.
// allow_pages = false keeps every decode call on the per-head kernel (whose split
// partials fit the allocation-free entry point's fixed workspace).
int fwd_impl(const tfa_fwd_params* a, void* workspace, size_t workspace_bytes, void* stream, void* ev_begin,
             void* ev_end, bool allow_pages);

// Byte ranges [off[i], off[i] + bytes[i]) of this call's workspace that must be zero
// when it starts (the control block and the decode kernel's split counters), and the
// workspace the call needs (*ws_bytes, if not null), for the plan fwd_impl makes with the
// same allow_pages.
int workspace_zero_ranges(const tfa_fwd_params* p, int device, size_t off[2], size_t bytes[2], bool allow_pages,
                          size_t* ws_bytes);

}  // namespace tfa
