// Plain C++ definitions shared by host-only (binding) and device code.
#pragma once

namespace cob {
enum DType : int { kF32 = 0, kF16 = 1, kBF16 = 2 };
}  // namespace cob
