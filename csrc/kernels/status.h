// Per-device status word that kernels set (atomicCAS from 0) when a bounded wait gives up.
#pragma once
#include <stdint.h>

namespace br {
int* status_ptr(int device);
}
