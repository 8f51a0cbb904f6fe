// Host-visible declarations of the packed-embedding codec (codec.cu); the C
// ABI is in include/wc_codec.h.
#pragma once
#include <stdint.h>

#include "../../include/wc_codec.h"
#include "../../include/wc_t5cuda.h"
