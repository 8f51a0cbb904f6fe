// Host-visible declarations of the query scoring kernel (query.cu); the C ABI
// is in include/wc_query.h.
#pragma once
#include "../../include/wc_query.h"
#include "../../include/wc_t5cuda.h"
