// Pre-included when build_ref_v8.py compiles the reference's v8 op (never by this
// repository's own code). With GCC >= 13 glibc spells M_LOG2Ef32 as a _Float32 literal
// (1.44...f32), which nvcc 12.9's device code generator rejects ("unsupported float
// variant"); math.h is included here first, so its include guard keeps later includes
// from redefining the constant, which is restated as an ordinary float literal.
#pragma once
#include <math.h>
#undef M_LOG2Ef32
#define M_LOG2Ef32 1.442695040888963407359924681001892137f
