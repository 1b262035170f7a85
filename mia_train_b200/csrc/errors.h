// Per-device error word shared by every kernel of the extension: a kernel whose bounded wait
// expires writes a nonzero code (first error wins, see common.cuh) and returns. The host reads and
// clears it with `check_errors()`, after a synchronisation point of its choosing.
#pragma once

#include <torch/extension.h>

namespace mia {

int* error_word(int device);
int64_t read_and_clear_errors(int64_t device);

}  // namespace mia
