// Host-only declarations shared with the binding files (which do not include device headers).
#pragma once

namespace cob {
// Process-wide programmatic-dependent-launch switch (see launch_k in common.cuh).
bool& pdl_flag();
// Process-wide count of weight tiles a GEMM prefetches into L2 beyond its ring (see common.cuh).
int& l2_prefetch_tiles();
}  // namespace cob
