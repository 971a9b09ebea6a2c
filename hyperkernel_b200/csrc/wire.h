// Request-ring wire format shared by the host encoder (device.cu, hk_encode_share) and the
// device decoder (the apply kernel in device.cu).
//
// A slot is [u32 message id | 12 bytes unused | body], 16 + the widest body rounded up to 16
// bytes, as Ring::push lays slots out (src/gpu/ring.rs:46-66: id at byte 0, body at
// RingConfig.body = 16).  Bodies carry the fields Feed::command writes per command
// (src/gpu/feed.rs:40-103); their byte sizes are the manifests' (end 8, pages 32, seat 52,
// prompt 40, start 56).  Span fields are {u64 address, u64 elements}; in this build the
// address is a byte offset from the start of the encoded stream, whose side blocks (Pages
// rows, Prompt tokens) follow the slots.
#pragma once

#include <stdint.h>

namespace hk {
namespace wire {

enum : uint32_t {
  kIdEnd = 0x101,
  kIdPages = 0x102,
  kIdSeat = 0x103,
  kIdPrompt = 0x104,
  kIdStart = 0x105,
};

constexpr uint32_t kBodyAt = 16;
constexpr uint32_t kWidest = 56;
constexpr uint32_t kSlot = (kBodyAt + kWidest + 15) / 16 * 16;  // 80

// end (8 B)
constexpr uint32_t kEndAt = 0, kEndLane = 4, kEndBytes = 8;
// pages (32 B)
constexpr uint32_t kPagesAt = 0, kPagesLane = 4, kPagesFrom = 8, kPagesUpto = 12, kPagesRow = 16,
                   kPagesBytes = 32;
// seat (52 B)
constexpr uint32_t kSeatAt = 0, kSeatLane = 4, kSeatPos = 8, kSeatBack = 12, kSeatSlot = 24,
                   kSeatTemp = 28, kSeatSeedLo = 32, kSeatSeedHi = 36, kSeatTopP = 40,
                   kSeatTopK = 44, kSeatLogprobs = 48, kSeatBytes = 52;
// prompt (40 B)
constexpr uint32_t kPromptLane = 0, kPromptLens = 4, kPromptTokens = 8, kPromptLps = 24,
                   kPromptBytes = 40;
// start (56 B)
constexpr uint32_t kStartAt = 0, kStartLane = 4, kStartNoise = 8, kStartIdle = 12,
                   kStartScratch = 16, kStartLps = 24, kStartCommits = 40, kStartBytes = 56;

static_assert(kStartBytes == kWidest, "the widest body sets the slot size");

}  // namespace wire
}  // namespace hk
