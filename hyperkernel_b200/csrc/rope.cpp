// RoPE cos/sin table for the MLA rope half (64 dims), built on the host with single-
// precision libm calls in the same order as the reference's table builder
// (src/gpu/load.rs:824-846): freq_i = 1 / base^(2i/dim), optional YaRN-style correction
// between the beta_fast / beta_slow rotation counts, then per row p the dim/2 cosines and
// dim/2 sines of p * freq_i.  Compiled with -ffp-contract=off so no step fuses into an
// fma; the table is pinned bit for bit against the reference's fixture windows.
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

#include "../../include/hk.h"

extern "C" int hk_rope_table(int64_t rows, int32_t dim, float base, int32_t original_seq_len,
                             float factor, float beta_fast, float beta_slow, float* table) {
  if (table == nullptr || rows < 0 || dim <= 0 || dim % 2 != 0 || dim > 4096) return HK_EINVAL;
  const int half = dim / 2;
  float* freqs = (float*)malloc(sizeof(float) * half);
  if (freqs == nullptr) return HK_ESPACE;
  for (int i = 0; i < half; ++i) freqs[i] = 1.0f / powf(base, (float)(2 * i) / (float)dim);
  if (original_seq_len > 0) {
    const float pi = 3.14159265358979323846f;
    auto corrected = [&](float rotations) {
      return (float)dim * logf((float)original_seq_len / (rotations * 2.0f * pi)) /
             (2.0f * logf(base));
    };
    const float low = fmaxf(floorf(corrected(beta_fast)), 0.0f);
    const float high = fminf(ceilf(corrected(beta_slow)), (float)dim - 1.0f);
    for (int i = 0; i < half; ++i) {
      float ramp = ((float)i - low) / fmaxf(high - low, 1e-3f);
      ramp = fminf(fmaxf(ramp, 0.0f), 1.0f);
      const float smooth = 1.0f - ramp;
      const float f = freqs[i];
      freqs[i] = f / factor * (1.0f - smooth) + f * smooth;
    }
  }
  for (int64_t p = 0; p < rows; ++p) {
    float* row = table + p * dim;
    for (int i = 0; i < half; ++i) {
      const float a = (float)p * freqs[i];
      row[i] = cosf(a);
      row[half + i] = sinf(a);
    }
  }
  free(freqs);
  return HK_OK;
}
