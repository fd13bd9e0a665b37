// Definitions of the opaque handle types shared by the C-ABI translation units.
#pragma once

#include <stdint.h>

struct kb_int8_weight {
  int device = 0;
  int n = 0, k = 0, kp = 0, n_stored = 0, layout = 0;
  int8_t* q = nullptr;
  float* scales = nullptr;
};
