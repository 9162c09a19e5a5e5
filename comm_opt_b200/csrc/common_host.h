// Host-only declarations shared with the binding files (which do not include device headers).
#pragma once

namespace cob {
// Process-wide programmatic-dependent-launch switch (see launch_k in common.cuh).
bool& pdl_flag();
}  // namespace cob
