/*
 * hk_oracle.c — CPU restatement of the decode step, used ONLY as the checker by tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg.  It is test infrastructure:
 * nothing in the product links or calls it.
 *
 * The reference (mr-d-self-driving/Hyperkernel) runs this step inside closed sm_103a cubins
 * with no source, so the numerics here come from the mathematics of each step; the index
 * semantics come from the reference's host code and tests:
 *   - pack / slot mapping: a row at position p of a lane lives in page row[p / page_rows],
 *     row p % page_rows (tests/engine.rs:105-113 Fake::write, :115-128 Fake::token), page 0
 *     is the scratch page that real rows never use (tests/engine.rs:108), block-table rows
 *     are Cache::pages output (src/engine/cache.rs:195-226);
 *   - the spec-verify block: 1 + drafts rows per lane per step (tests/engine.rs:173-193);
 *   - RoPE table: src/gpu/load.rs:824-846, pinned against tests/fixtures/rope.json.
 * Parity status: pack / append / route ids / permutation / rope are pinned bit-exact
 * (rope against the reference's fixture bytes); attention, GEMM and MoE numerics are
 * "parity unpinned" against the reference (no reference test pins them) and are checked
 * against this fp64-accumulated restatement within the stated tolerances.
 *
 * Build: oracle/build.py (gcc -O2 -fopenmp -ffp-contract=off -> oracle/_build/liboracle.so).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------------------------- */
/* number formats                                                                      */
/* ---------------------------------------------------------------------------------- */

static float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

uint16_t orc_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* e4m3 (OCP FP8, bias 7, no infinities, max 448): decode is exact. */
float orc_e4m3_to_f32(uint8_t v) {
  int s = v >> 7, e = (v >> 3) & 15, m = v & 7;
  float r;
  if (e == 15 && m == 7) return NAN;
  if (e == 0) r = ldexpf((float)m, -9);
  else r = ldexpf(1.0f + (float)m / 8.0f, e - 7);
  return s ? -r : r;
}

/* Round to nearest even with saturation to +-448 (the satfinite conversion). */
uint8_t orc_f32_to_e4m3(float f) {
  if (isnan(f)) return 0x7f;
  uint8_t sign = signbit(f) ? 0x80 : 0;
  float a = fabsf(f);
  if (a >= 448.0f) return sign | 0x7e;
  if (a < ldexpf(1.0f, -6)) { /* subnormal: multiples of 2^-9 */
    float q = rintf(ldexpf(a, 9));
    int m = (int)q;
    if (m >= 8) return sign | 0x08;
    return sign | (uint8_t)m;
  }
  int e;
  float fr = frexpf(a, &e); /* a = fr * 2^e, fr in [0.5, 1) */
  e -= 1;                   /* a = (2 fr) * 2^e, 2fr in [1, 2) */
  float mant = ldexpf(fr, 1) - 1.0f;
  int m = (int)rintf(mant * 8.0f);
  if (m == 8) {
    m = 0;
    e += 1;
  }
  int be = e + 7;
  if (be > 15 || (be == 15 && m == 7)) return sign | 0x7e;
  return sign | (uint8_t)((be << 3) | m);
}

/* The deterministic sigmoid of the router (same fmaf sequence as the device code). */
static float exp_det(float y) {
  if (y > 88.0f) y = 88.0f;
  if (y < -87.0f) y = -87.0f;
  const float kLog2e = 1.44269504088896341f;
  float t = y * kLog2e;
  float n = rintf(t);
  float r = t - n;
  const float c1 = 0.693147180559945309f, c2 = 0.240226506959100712f,
              c3 = 0.0555041086648215800f, c4 = 0.00961812910762847717f,
              c5 = 0.00133335581464284434f, c6 = 0.000154035303933816099f,
              c7 = 0.0000152527338040598403f;
  float p = c7;
  p = fmaf(p, r, c6);
  p = fmaf(p, r, c5);
  p = fmaf(p, r, c4);
  p = fmaf(p, r, c3);
  p = fmaf(p, r, c2);
  p = fmaf(p, r, c1);
  p = fmaf(p, r, 1.0f);
  return ldexpf(p, (int)n);
}

float orc_sigmoid(float x) { return 1.0f / (1.0f + exp_det(-x)); }

/* ---------------------------------------------------------------------------------- */
/* a7 pack                                                                             */
/* ---------------------------------------------------------------------------------- */

/* Returns the number of rows T; *err = 0 when clean, else the first error code
 * (1 overflow, 2 a row through the scratch page or past the pool). */
int orc_pack(const int32_t* lane_tokens, const int32_t* lane_pos, const int32_t* bt,
             int bt_stride, int num_lanes, int page_size, int num_pages, int max_tokens,
             int32_t* cu, int32_t* seq_lens, int32_t* positions, int32_t* slot,
             int32_t* token_lane, int32_t* active, int* err) {
  int run = 0, na = 0;
  *err = 0;
  for (int b = 0; b < num_lanes; ++b) {
    int n = lane_tokens[b] > 0 ? lane_tokens[b] : 0;
    cu[b] = run;
    seq_lens[b] = n > 0 ? lane_pos[b] + n : 0;
    if (n > 0) active[1 + na++] = b;
    run += n;
  }
  cu[num_lanes] = run;
  active[0] = na;
  if (run > max_tokens && *err == 0) *err = 1;
  for (int b = 0; b < num_lanes; ++b) {
    for (int j = 0; j < lane_tokens[b]; ++j) {
      int t = cu[b] + j;
      if (t >= max_tokens) continue;
      int pos = lane_pos[b] + j, blk = pos / page_size;
      int page = (pos >= 0 && blk < bt_stride) ? bt[(int64_t)b * bt_stride + blk] : -1;
      int s;
      if (page <= 0 || page >= num_pages) {
        if (*err == 0) *err = 2;
        s = -1;
      } else {
        s = page * page_size + pos % page_size;
      }
      positions[t] = pos;
      slot[t] = s;
      token_lane[t] = b;
    }
  }
  return run;
}

/* ---------------------------------------------------------------------------------- */
/* a8 KV append                                                                        */
/* ---------------------------------------------------------------------------------- */

/* Offset of element (slot, e) of a latent cache: row-major when page_rows == 0, else the
 * page-blocked layout (pages of page_rows rows, each storing its rows in blocks of 64
 * elements, block-major) that the device's latent cache uses. */
static int64_t latent_off(int64_t slot, int e, int row, int page_rows) {
  if (page_rows == 0) return slot * row + e;
  return (slot / page_rows) * page_rows * row + (int64_t)(e / 64) * page_rows * 64 +
         (slot % page_rows) * 64 + e % 64;
}

int orc_kv_append_u16(const uint16_t* src, const int32_t* slot, int T, int row, int page_rows,
                      uint16_t* cache, int64_t num_slots) {
  int err = 0;
  for (int t = 0; t < T; ++t) {
    if (slot[t] < 0 || slot[t] >= num_slots) {
      err = 3;
      continue;
    }
    for (int e = 0; e < row; ++e) cache[latent_off(slot[t], e, row, page_rows)] = src[(int64_t)t * row + e];
  }
  return err;
}

int orc_kv_append_f32(const float* k, const float* v, const int32_t* slot, int T, int row,
                      float* kc, float* vc, int64_t num_slots) {
  int err = 0;
  for (int t = 0; t < T; ++t) {
    if (slot[t] < 0 || slot[t] >= num_slots) {
      err = 3;
      continue;
    }
    memcpy(kc + (int64_t)slot[t] * row, k + (int64_t)t * row, sizeof(float) * row);
    memcpy(vc + (int64_t)slot[t] * row, v + (int64_t)t * row, sizeof(float) * row);
  }
  return err;
}

/* Row quantisation: scale = max(amax, 1e-12) / 448, q = e4m3(x / scale). */
int orc_kv_append_fp8(const uint16_t* src, const int32_t* slot, int T, int row, uint8_t* cache,
                      float* scales, int64_t num_slots) {
  int err = 0;
  for (int t = 0; t < T; ++t) {
    if (slot[t] < 0 || slot[t] >= num_slots) {
      err = 3;
      continue;
    }
    float amax = 0.f;
    for (int i = 0; i < row; ++i) amax = fmaxf(amax, fabsf(bf16_to_f32(src[(int64_t)t * row + i])));
    float s = fmaxf(amax, 1e-12f) / 448.0f;
    for (int i = 0; i < row; ++i)
      cache[(int64_t)slot[t] * row + i] = orc_f32_to_e4m3(bf16_to_f32(src[(int64_t)t * row + i]) / s);
    scales[slot[t]] = s;
  }
  return err;
}

/* ---------------------------------------------------------------------------------- */
/* a9 attention                                                                        */
/* ---------------------------------------------------------------------------------- */

static int lane_of(const int32_t* cu, int num_lanes, int t) {
  int b = 0;
  while (b + 1 < num_lanes && cu[b + 1] <= t) ++b;
  return b;
}

/* GQA fp32: fp64 accumulation of scores and values. */
void orc_gqa_decode_f32(const float* q, const float* kc, const float* vc, const int32_t* bt,
                        int bt_stride, const int32_t* cu, const int32_t* positions, int num_lanes,
                        int T, int qh, int kvh, int D, int page_size, float scale, float* out,
                        float* lse) {
  const int group = qh / kvh;
#pragma omp parallel for collapse(2) schedule(dynamic)
  for (int t = 0; t < T; ++t) {
    for (int h = 0; h < qh; ++h) {
      const int b = lane_of(cu, num_lanes, t), pos = positions[t], g = h / group;
      double* s = (double*)malloc(sizeof(double) * (pos + 1));
      double m = -INFINITY;
      for (int p = 0; p <= pos; ++p) {
        int64_t slot = (int64_t)bt[(int64_t)b * bt_stride + p / page_size] * page_size + p % page_size;
        const float* k = kc + (slot * kvh + g) * D;
        double acc = 0;
        for (int d = 0; d < D; ++d) acc += (double)q[((int64_t)t * qh + h) * D + d] * k[d];
        s[p] = acc * scale;
        if (s[p] > m) m = s[p];
      }
      double l = 0;
      double* o = (double*)calloc(D, sizeof(double));
      for (int p = 0; p <= pos; ++p) {
        int64_t slot = (int64_t)bt[(int64_t)b * bt_stride + p / page_size] * page_size + p % page_size;
        const float* v = vc + (slot * kvh + g) * D;
        double w = exp(s[p] - m);
        l += w;
        for (int d = 0; d < D; ++d) o[d] += w * v[d];
      }
      for (int d = 0; d < D; ++d) out[((int64_t)t * qh + h) * D + d] = (float)(o[d] / l);
      lse[(int64_t)t * qh + h] = (float)(m + log(l));
      free(o);
      free(s);
    }
  }
}

/* MLA absorbed attention over a page-blocked bf16 latent cache (kv_fp8 == NULL; blocks of 64
 * elements in pages of page_size rows) or a row-major e4m3*scale latent cache.
 * Query row t attends KV rows [max(0, kv_begin[b]), min(positions[t] + 1, kv_end[b]))
 * (kv_begin / kv_end may be NULL: the whole causal prefix).  Scores over 576 dims, values
 * the first 512, fp64 accumulation; out[T][heads][512] fp32, lse[T][heads]. */
void orc_mla_decode(const uint16_t* q, const uint16_t* kv_bf16, const uint8_t* kv_fp8,
                    const float* kv_scale, const int32_t* bt, int bt_stride, const int32_t* cu,
                    const int32_t* positions, const int32_t* kv_begin, const int32_t* kv_end,
                    int num_lanes, int T, int heads, int page_size, float scale, float* out,
                    float* lse) {
  const int DK = 576, DV = 512;
  /* Rows of the query block of one lane share their KV: convert it once per row t, then
   * spread the heads over the threads. */
  for (int t = 0; t < T; ++t) {
    const int b = lane_of(cu, num_lanes, t);
    int lo = 0, hi = positions[t] + 1;
    if (kv_begin) {
      if (kv_begin[b] > lo) lo = kv_begin[b];
      if (kv_end[b] < hi) hi = kv_end[b];
    }
    const int n = hi > lo ? hi - lo : 0;
    float* k = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1) * DK);
#pragma omp parallel for schedule(static)
    for (int j = 0; j < n; ++j) {
      const int p = lo + j;
      const int64_t slot =
          (int64_t)bt[(int64_t)b * bt_stride + p / page_size] * page_size + p % page_size;
      for (int d = 0; d < DK; ++d)
        k[(int64_t)j * DK + d] = kv_fp8 ? orc_e4m3_to_f32(kv_fp8[slot * DK + d]) * kv_scale[slot]
                                        : bf16_to_f32(kv_bf16[latent_off(slot, d, DK, page_size)]);
    }
#pragma omp parallel for schedule(dynamic)
    for (int h = 0; h < heads; ++h) {
      double* s = (double*)malloc(sizeof(double) * (size_t)(n > 0 ? n : 1));
      double* o = (double*)malloc(sizeof(double) * DV);
      float qf[576];
      const int64_t row = (int64_t)t * heads + h;
      for (int d = 0; d < DK; ++d) qf[d] = bf16_to_f32(q[row * DK + d]);
      double m = -INFINITY;
      for (int j = 0; j < n; ++j) {
        double acc = 0;
        const float* kr = k + (int64_t)j * DK;
        for (int d = 0; d < DK; ++d) acc += (double)qf[d] * kr[d];
        s[j] = acc * scale;
        if (s[j] > m) m = s[j];
      }
      double l = 0;
      for (int d = 0; d < DV; ++d) o[d] = 0;
      for (int j = 0; j < n; ++j) {
        const double w = exp(s[j] - m);
        l += w;
        const float* kr = k + (int64_t)j * DK;
        for (int d = 0; d < DV; ++d) o[d] += w * kr[d];
      }
      for (int d = 0; d < DV; ++d) out[row * DV + d] = n > 0 ? (float)(o[d] / l) : 0.f;
      lse[row] = n > 0 ? (float)(m + log(l)) : -INFINITY;
      free(o);
      free(s);
    }
    free(k);
  }
}

/* a10 LSE merge of n partials o[n][rows][dv], lse[n][rows] -> out[rows][dv], lse_out. */
void orc_lse_merge(const float* o, const float* lse, int n, int64_t rows, int dv, float* out,
                   float* lse_out) {
#pragma omp parallel for
  for (int64_t r = 0; r < rows; ++r) {
    double m = -INFINITY;
    for (int p = 0; p < n; ++p)
      if (lse[(int64_t)p * rows + r] > m) m = lse[(int64_t)p * rows + r];
    double sum = 0;
    for (int p = 0; p < n; ++p) {
      const double lp = lse[(int64_t)p * rows + r];
      if (lp != -INFINITY) sum += exp(lp - m);
    }
    for (int d = 0; d < dv; ++d) {
      double acc = 0;
      for (int p = 0; p < n; ++p) {
        const double lp = lse[(int64_t)p * rows + r];
        if (lp != -INFINITY) acc += exp(lp - m) * o[((int64_t)p * rows + r) * dv + d];
      }
      out[r * dv + d] = sum > 0 ? (float)(acc / sum) : 0.f;
    }
    if (lse_out) lse_out[r] = sum > 0 ? (float)(m + log(sum)) : -INFINITY;
  }
}

/* ---------------------------------------------------------------------------------- */
/* a11 FP8 block-scaled linear                                                         */
/* ---------------------------------------------------------------------------------- */

void orc_quant_fp8(const uint16_t* x, int64_t rows, int k, uint8_t* xq, float* sx) {
  const int nb = k / 128;
#pragma omp parallel for
  for (int64_t r = 0; r < rows; ++r) {
    for (int kb = 0; kb < nb; ++kb) {
      float amax = 0.f;
      for (int i = 0; i < 128; ++i) amax = fmaxf(amax, fabsf(bf16_to_f32(x[r * k + kb * 128 + i])));
      const float s = fmaxf(amax, 1e-12f) / 448.0f;
      for (int i = 0; i < 128; ++i)
        xq[r * k + kb * 128 + i] = orc_f32_to_e4m3(bf16_to_f32(x[r * k + kb * 128 + i]) / s);
      sx[r * nb + kb] = s;
    }
  }
}

/* y[m][n] = sum_kb (sum_k xq wq) * sx[m][kb] * sw[n/128][kb], fp64 accumulation. */
void orc_gemm_fp8(const uint8_t* xq, const float* sx, const uint8_t* wq, const float* sw,
                  int64_t m, int n, int k, float* y) {
  const int nb = k / 128;
  float lut[256];
  for (int i = 0; i < 256; ++i) lut[i] = orc_e4m3_to_f32((uint8_t)i);
#pragma omp parallel for schedule(dynamic)
  for (int64_t r = 0; r < m; ++r) {
    for (int c = 0; c < n; ++c) {
      double acc = 0;
      for (int kb = 0; kb < nb; ++kb) {
        double part = 0;
        const uint8_t* a = xq + r * k + kb * 128;
        const uint8_t* b = wq + (int64_t)c * k + kb * 128;
        for (int i = 0; i < 128; ++i) part += (double)lut[a[i]] * lut[b[i]];
        acc += part * sx[r * nb + kb] * sw[(int64_t)(c / 128) * nb + kb];
      }
      y[r * n + c] = (float)acc;
    }
  }
}

/* ---------------------------------------------------------------------------------- */
/* a12-a15 MoE                                                                         */
/* ---------------------------------------------------------------------------------- */

/* Sigmoid router: top_k of s + bias (ties: lower expert id), weights s / sum(s) * scale
 * with the sum taken in selection order. */
void orc_route(const float* logits, const float* bias, int tokens, int E, int top_k,
               float route_scale, int32_t* ids, float* weights) {
  for (int t = 0; t < tokens; ++t) {
    float s[1024], sel[1024];
    for (int e = 0; e < E; ++e) {
      s[e] = orc_sigmoid(logits[(int64_t)t * E + e]);
      sel[e] = s[e] + (bias ? bias[e] : 0.f);
    }
    float sum = 0.f, chosen[64];
    for (int k = 0; k < top_k; ++k) {
      int best = -1;
      for (int e = 0; e < E; ++e)
        if (sel[e] != -INFINITY && (best < 0 || sel[e] > sel[best])) best = e;
      ids[(int64_t)t * top_k + k] = best;
      chosen[k] = s[best];
      sum += s[best];
      sel[best] = -INFINITY;
    }
    for (int k = 0; k < top_k; ++k) weights[(int64_t)t * top_k + k] = (chosen[k] / sum) * route_scale;
  }
}

/* Stable counting sort of (token, k) pairs by expert. */
void orc_permute(const int32_t* ids, const float* weights, int tokens, int top_k, int E,
                 int32_t* offsets, int32_t* perm_token, float* perm_weight, int32_t* inv) {
  const int P = tokens * top_k;
  int* cnt = (int*)calloc(E + 1, sizeof(int));
  for (int p = 0; p < P; ++p) cnt[ids[p]]++;
  int run = 0;
  for (int e = 0; e < E; ++e) {
    offsets[e] = run;
    run += cnt[e];
    cnt[e] = offsets[e];
  }
  offsets[E] = run;
  for (int p = 0; p < P; ++p) {
    const int dst = cnt[ids[p]]++;
    perm_token[dst] = p / top_k;
    perm_weight[dst] = weights[p];
    inv[p] = dst;
  }
  free(cnt);
}

/* Grouped expert FFN with the device's quantisation points: g, u fp64-accumulated per
 * 128-block and scaled, h = silu(g) * u rounded to fp32, requantised to e4m3 1x128, then
 * the down projection.  y[P][hidden] fp32. */
void orc_moe_grouped(const uint8_t* xq, const float* sx, const int32_t* offsets,
                     const int32_t* perm_token, int E, int hidden, int inter, const uint8_t* w13,
                     const float* s13, const uint8_t* w2, const float* s2, float* y) {
  float lut[256];
  for (int i = 0; i < 256; ++i) lut[i] = orc_e4m3_to_f32((uint8_t)i);
  const int kbh = hidden / 128, kbi = inter / 128;
  const int P = offsets[E];
  int* expert_of = (int*)malloc(sizeof(int) * (P > 0 ? P : 1));
  for (int e = 0; e < E; ++e)
    for (int p = offsets[e]; p < offsets[e + 1]; ++p) expert_of[p] = e;
#pragma omp parallel for schedule(dynamic)
  for (int p = 0; p < P; ++p) {
    const int e = expert_of[p], src = perm_token[p];
    const uint8_t* x = xq + (int64_t)src * hidden;
    const uint8_t* wg = w13 + (int64_t)e * 2 * inter * hidden;
    const uint8_t* wu = wg + (int64_t)inter * hidden;
    const float* sg = s13 + (int64_t)e * (2 * inter / 128) * kbh;
    const float* su = sg + (int64_t)(inter / 128) * kbh;
    float* h = (float*)malloc(sizeof(float) * inter);
    uint8_t* hq = (uint8_t*)malloc(inter);
    float* hs = (float*)malloc(sizeof(float) * kbi);
    for (int j = 0; j < inter; ++j) {
      double g = 0, u = 0;
      for (int kb = 0; kb < kbh; ++kb) {
        double pg = 0, pu = 0;
        for (int i = 0; i < 128; ++i) {
          const double a = lut[x[kb * 128 + i]];
          pg += a * lut[wg[(int64_t)j * hidden + kb * 128 + i]];
          pu += a * lut[wu[(int64_t)j * hidden + kb * 128 + i]];
        }
        const double xs = sx[(int64_t)src * kbh + kb];
        g += pg * xs * sg[(int64_t)(j / 128) * kbh + kb];
        u += pu * xs * su[(int64_t)(j / 128) * kbh + kb];
      }
      h[j] = (float)(g / (1.0 + exp(-g)) * u);
    }
    for (int kb = 0; kb < kbi; ++kb) {
      float amax = 0.f;
      for (int i = 0; i < 128; ++i) amax = fmaxf(amax, fabsf(h[kb * 128 + i]));
      const float s = fmaxf(amax, 1e-12f) / 448.0f;
      hs[kb] = s;
      for (int i = 0; i < 128; ++i) hq[kb * 128 + i] = orc_f32_to_e4m3(h[kb * 128 + i] / s);
    }
    const uint8_t* wd = w2 + (int64_t)e * hidden * inter;
    const float* sd = s2 + (int64_t)e * (hidden / 128) * kbi;
    for (int c = 0; c < hidden; ++c) {
      double acc = 0;
      for (int kb = 0; kb < kbi; ++kb) {
        double part = 0;
        for (int i = 0; i < 128; ++i)
          part += (double)lut[hq[kb * 128 + i]] * lut[wd[(int64_t)c * inter + kb * 128 + i]];
        acc += part * hs[kb] * sd[(int64_t)(c / 128) * kbi + kb];
      }
      y[(int64_t)p * hidden + c] = (float)acc;
    }
    free(hs);
    free(hq);
    free(h);
  }
  free(expert_of);
}

/* out[t] = sum_k perm_weight[inv[t,k]] * y[inv[t,k]] (+ shared[t]); y, shared bf16. */
void orc_combine(const uint16_t* y, const float* perm_weight, const int32_t* inv,
                 const uint16_t* shared, int tokens, int top_k, int hidden, float* out) {
#pragma omp parallel for
  for (int t = 0; t < tokens; ++t) {
    for (int d = 0; d < hidden; ++d) {
      double acc = 0;
      for (int k = 0; k < top_k; ++k) {
        const int r = inv[(int64_t)t * top_k + k];
        acc += (double)perm_weight[r] * bf16_to_f32(y[(int64_t)r * hidden + d]);
      }
      if (shared) acc += bf16_to_f32(shared[(int64_t)t * hidden + d]);
      out[(int64_t)t * hidden + d] = (float)acc;
    }
  }
}

/* ---------------------------------------------------------------------------------- */
/* RoPE table (src/gpu/load.rs:824-846)                                                */
/* ---------------------------------------------------------------------------------- */

void orc_rope_table(int64_t rows, int dim, float base, int original_seq_len, float factor,
                    float beta_fast, float beta_slow, float* table) {
  const int half = dim / 2;
  float freqs[2048];
  for (int i = 0; i < half; ++i) freqs[i] = 1.0f / powf(base, (float)(2 * i) / (float)dim);
  if (original_seq_len > 0) {
    const float pi = 3.14159265358979323846f;
    float c_fast = (float)dim * logf((float)original_seq_len / (beta_fast * 2.0f * pi)) / (2.0f * logf(base));
    float c_slow = (float)dim * logf((float)original_seq_len / (beta_slow * 2.0f * pi)) / (2.0f * logf(base));
    float low = fmaxf(floorf(c_fast), 0.0f);
    float high = fminf(ceilf(c_slow), (float)dim - 1.0f);
    for (int i = 0; i < half; ++i) {
      float ramp = ((float)i - low) / fmaxf(high - low, 1e-3f);
      ramp = fminf(fmaxf(ramp, 0.0f), 1.0f);
      float smooth = 1.0f - ramp;
      freqs[i] = freqs[i] / factor * (1.0f - smooth) + freqs[i] * smooth;
    }
  }
#pragma omp parallel for
  for (int64_t p = 0; p < rows; ++p) {
    for (int i = 0; i < half; ++i) {
      float a = (float)p * freqs[i];
      table[p * dim + i] = cosf(a);
      table[p * dim + half + i] = sinf(a);
    }
  }
}

/* Sets the OpenMP thread count of later calls (a launcher may have set OMP_NUM_THREADS=1). */
int orc_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
#else
  (void)n;
  return 1;
#endif
}

int orc_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
