// Flash-attention forward for sm_100a (placeholder entry point until the kernel lands).
#include "lumen_b200_internal.h"

extern "C" int lumen_b200_fa_fwd_bf16(const void*, const void*, const void*, void*, int, int, int,
                                       int, int, float, int, void*) {
  return LUMEN_B200_EUNSUPPORTED;
}
