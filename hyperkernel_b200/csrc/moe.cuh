// Internal interface of the grouped MoE FFN launchers (moe.cu, moe_sm100.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace hk {

// Row-tile widths of the tensor-core path (the MMA's N), one chosen per call from the rows its
// experts hold on average (at least the width's threshold): 16 (below 8), 32 (8-23), 64
// (24-55), 96 (56 and up).  Narrower tiles leave room for more stages of weights in flight;
// 96 rows is the most each promotion thread's gate and up sums (half a tile's rows each) fit
// in 168 registers, what a 320-thread CTA's threads get (three warps of a sub-partition share
// its 16,384).
__host__ __device__ constexpr int moe_tile_width(int i) { return i == 0 ? 16 : i == 1 ? 32 : i == 2 ? 64 : 96; }
__host__ __device__ constexpr int moe_tile_min_avg(int i) { return i == 0 ? 0 : i == 1 ? 8 : i == 2 ? 24 : 56; }

// Scratch of one grouped-FFN call, carved from the caller's workspace:
//   hq [rows][inter] e4m3, hs [rows][inter/128], the portable kernels' tile list (64-row
//   tiles), then xp [rows][hidden] e4m3, sxp [rows][hidden/128] and the tensor-core kernels'
//   tile list (tiles of the chosen width, room for 16-row tiles) with its width word.
struct MoeScratch {
  uint8_t* hq;
  float* hs;
  int32_t* tile_expert;
  int32_t* tile_row;
  int32_t* num_tiles;
  int32_t max_tiles;
  uint8_t* xp;
  float* sxp;
  int32_t* tc_expert;
  int32_t* tc_row;
  int32_t* tc_num;   // [0] tiles, [1] their width
  int32_t max_tc;
};

// Bytes of the portable kernels' scratch (hq, hs, tile list): a prefix of the full layout.
size_t moe_portable_workspace(int64_t rows, int32_t inter);
// Bytes of the full layout (what hk_moe_workspace_size returns).
size_t moe_full_workspace(int64_t rows, int32_t hidden, int32_t inter);

// hk_moe_grouped's launcher with the device error word passed in (nullptr: bad rows are
// skipped without being recorded).  portable_only selects the CUDA-core kernels, whose
// scratch is the moe_portable_workspace prefix.
int moe_grouped_run(const uint8_t* xq, const float* sx, int32_t tokens, const int32_t* offsets,
                    const int32_t* perm_token, int64_t rows, int32_t num_experts, int32_t hidden,
                    int32_t inter, const uint8_t* w13, const float* s13, const uint8_t* w2,
                    const float* s2, uint16_t* y, void* workspace, size_t workspace_bytes,
                    bool portable_only, unsigned long long* err, cudaStream_t s);

bool moe_sm100_supported(int32_t num_experts, int32_t hidden, int32_t inter);

int moe_sm100_run(const uint8_t* xq, const float* sx, int32_t tokens, const int32_t* offsets,
                  const int32_t* perm_token, int64_t rows, int32_t num_experts, int32_t hidden, int32_t inter,
                  const uint8_t* w13, const float* s13, const uint8_t* w2, const float* s2, uint16_t* y,
                  const MoeScratch& ws, int widths, unsigned long long* err, cudaStream_t s);

}  // namespace hk
