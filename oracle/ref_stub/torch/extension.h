/* TEST INFRASTRUCTURE ONLY.  Stand-in for <torch/extension.h> when the
 * reference's csrc/transfer.cu is compiled as the GPU oracle: that file
 * includes the torch header but uses nothing from it except the fixed-width
 * integer types, so the oracle build needs no libtorch. */
#pragma once
#include <cstdint>
#include <cstddef>
