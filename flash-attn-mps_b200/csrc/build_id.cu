// Build identity of the library: the hash of every compiled source, header
// and compiler flag, computed by build.py (source_hash) and passed in as
// FAB_BUILD_ID when this file is compiled. build.py recompiles this file
// whenever that hash changes, so the value always describes the sources the
// library was linked from.
#include "flash_attn_b200.h"

#ifndef FAB_BUILD_ID
#define FAB_BUILD_ID "unknown"
#endif

extern "C" const char* fa_build_id(void) { return FAB_BUILD_ID; }
