// Internal interface of the grouped MoE FFN launchers (moe.cu, moe_sm100.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace hk {

// Rows of the tensor-core path's wide row tiles (the MMA's N).  Each promotion thread keeps
// gate and up sums for half of a tile's rows, and 96 rows is what 168 registers a thread (the
// most a 320-thread CTA gets: three warps of a sub-partition share its 16,384) hold without
// spilling; the narrow tiles have 64.
constexpr int kMoeWideRows = 96;

// Scratch of one grouped-FFN call, carved from the caller's workspace:
//   hq [rows][inter] e4m3, hs [rows][inter/128], the tile list (the portable kernels' 64-row
//   tiles, or the tcgen05 kernels' narrow tiles), then xp [rows][hidden] e4m3,
//   sxp [rows][hidden/128] and the wide (kMoeWideRows-row) tile list (tcgen05 only).
struct MoeScratch {
  uint8_t* hq;
  float* hs;
  int32_t* tile_expert;
  int32_t* tile_row;
  int32_t* num_tiles;
  int32_t max_tiles;
  uint8_t* xp;
  float* sxp;
  int32_t* wide_expert;
  int32_t* wide_row;
  int32_t* num_wide;
  int32_t max_wide;
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
                  const MoeScratch& ws, bool wide, unsigned long long* err, cudaStream_t s);

}  // namespace hk
