// Host-side helpers shared between the C-ABI translation units.
#pragma once

#include <cstddef>

#include "../../include/tfa.h"

namespace tfa {

// The forward used by tfa_fwd / tfa_fwd_timed: validation, split-KV plan, TMA
// descriptors and launches on `stream`, with the caller's workspace. ev_begin / ev_end
// (cudaEvent_t or NULL) are recorded around the attention kernel.
int fwd_impl(const tfa_fwd_params* a, void* workspace, size_t workspace_bytes, void* stream, void* ev_begin,
             void* ev_end);

// Byte ranges [off[i], off[i] + bytes[i]) of this call's workspace that must be zero
// when it starts (the control block and the decode kernel's split counters).
int workspace_zero_ranges(const tfa_fwd_params* p, int device, size_t off[2], size_t bytes[2]);

}  // namespace tfa
