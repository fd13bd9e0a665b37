// Definitions of the opaque handle types shared by the C-ABI translation units.
#pragma once

#include <stddef.h>
#include <stdint.h>

struct kb_int8_weight {
  int device = 0;
  int n = 0, k = 0, kp = 0, n_stored = 0, layout = 0;
  int8_t* q = nullptr;
  float* scales = nullptr;
};

struct kb_mxfp8_weight {
  int device = 0;
  int n = 0, k = 0, kp = 0, blocks4 = 0;
  uint8_t* q = nullptr;       // E4M3 [n, kp]
  uint8_t* scales = nullptr;  // packed UE8M0 tiles
  size_t scale_bytes = 0;
};
