// Internal interface of the HK_MODEL_MLA decoder (model.cu) used by the device kernel
// behind hk_open / hk_push / hk_drain (device.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/hk.h"

namespace hk {

struct MlaLayer {
  uint8_t *wqa, *wqb, *wkva, *wo, *wr, *w13, *w2;
  float *sqa, *sqb, *skva, *so, *sr, *s13, *s2;
  uint16_t* kv;  // page-blocked latent cache, [pages * 64][576] bf16
};

// What one forward pass reads and where the sampled results go.  All pointers are device
// memory owned by MlaModel; the host fills the small per-step arrays through `stage`.
struct MlaModel {
  hk_mla_model dims{};
  int32_t width = 0, block = 0, page_rows = 0, context = 0, chunk = 0, entries = 0, bt_stride = 0;
  int64_t pages = 0;
  int32_t t_cap = 0;  // rows one forward pass takes
  int32_t r_cap = 0;  // rows one forward pass samples
  int32_t n_lp = 0;   // logprob pairs per sampled token
  uint16_t* embed = nullptr;
  uint8_t* wvocab = nullptr;
  float* svocab = nullptr;
  std::vector<MlaLayer> layers;
  // step buffers
  int32_t *lane_tokens, *lane_pos, *cu_seqlens, *seq_lens, *positions, *slots, *token_lane, *active;
  int32_t *tokens_in, *drafts, *gather, *cu_rows;
  uint16_t *x, *qa, *q, *kvn, *o, *y, *rl, *ym, *mo, *logits_bf16;
  uint8_t *xq, *qaq, *oq;
  float *xs, *qas, *os, *rlf, *logits, *lse;
  int32_t *ids_e, *perm_token, *inv, *offsets, *out_ids;
  float *w_e, *perm_w, *lp;
  hk_sampling* sampling;     // per lane, written by the Seat command
  uint64_t* state;           // per lane generator state, seeded by the Seat command
  int32_t* tok;              // per lane last token (the next decode row's input)
  void *attn_ws, *moe_ws, *sample_ws;
  size_t attn_ws_bytes = 0, moe_ws_bytes = 0, sample_ws_bytes = 0;
  int32_t* stage_h = nullptr;  // pinned host staging for the per-step uploads
  int32_t* stage_d = nullptr;
  size_t stage_words = 0;
  std::vector<void*> allocations;
};

// Checks the dimensions against the kernels' limits.
int mla_check(const hk_config& cfg, const hk_mla_model& m);
// Allocates and seeds the weights, the latent caches and the step buffers on the current
// device (zeroed caches); `rows` is the device block-table array [width][bt_stride].
int mla_create(const hk_config& cfg, const hk_mla_model& m, MlaModel** out, cudaStream_t s);
void mla_destroy(MlaModel* m);
int mla_tensor(MlaModel* m, int32_t* token_pool, size_t token_pool_bytes, uint32_t layer, const char* name,
               void** ptr, size_t* bytes);

// One lane's part of a forward pass.
struct MlaLaneRows {
  int32_t lane, pos, rows;
};

// The decode step: every lane in `lanes` runs `rows` rows from `pos` (its last token, then
// drafts found by prompt lookup in the token pool).  Writes out_ids [width][block] (accepted
// ids, then -2) and lp [width][block][2 n_lp + 1]; updates the lanes' last tokens.  `rows_dev`
// is the device block-table array [width][bt_stride], `pool` the token pool; a token-pool write
// through a bad page records its fault in `dev_err` (the handle's error words).
int mla_decode_step(MlaModel* m, const std::vector<MlaLaneRows>& lanes, const int32_t* rows_dev, int32_t* pool,
                    unsigned long long* dev_err, cudaStream_t s);
// A batch of prompt chunks of distinct lanes, lanes ascending, `tokens` their chunks in that
// order: the tokens are written to the token pool and prefilled; each lane is answered with a
// token sampled from its chunk's last row (out_ids[lane], lp [width][2 n_lp + 1]).
int mla_prompt_step(MlaModel* m, const std::vector<MlaLaneRows>& lanes, const std::vector<int32_t>& tokens,
                    const int32_t* rows_dev, int32_t* pool, unsigned long long* dev_err, cudaStream_t s);

}  // namespace hk
