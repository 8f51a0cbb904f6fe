// Host-visible declarations of the index-build kernels (index.cu); the C ABI
// is in include/wc_index.h.
#pragma once
#include "../../include/wc_index.h"
#include "../../include/wc_t5cuda.h"
