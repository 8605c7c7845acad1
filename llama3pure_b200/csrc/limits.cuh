// limits.cuh -- sizes shared by the kernels (the NVLink groups of
// seq_xchg.cuh and wo.cuh, the host-call server) and the host context (ctx.h).
#pragma once
#include <cstddef>

namespace l3p {

// The split-K scratch of a context (partials, (m, l) pairs, tickets) is used
// in this many rotating slices, so that decode launches overlapping on the
// GPU never share one; the host-call server uses slices 0 and 1 by call parity.
constexpr int kScratchSlots = 4;

// wo GEMV kernels: 14 weight formats x (4, 8 warps)
constexpr int kWoKernelCount = 28;

constexpr int kXchgMaxParts = 16;    // members of a sequence or tensor-parallel group
constexpr int kXchgFlagBytes = 256;  // flags and step counter ahead of an exchange region's slots

// Exchange region of a tensor-parallel group (wo.cuh), byte offsets:
//   [0, 256)        header: u32 step (calls completed) at 64, u32 exit ticket at 68
//   kTpRecvOff      u64 recv[2][n_members][dim]: every member's partial rows
// Every u64 is a packet: the float in the low 32 bits, the call number e in
// the high 32 (never 0: calls count from 1).  The slots alternate by call parity.
constexpr int kTpMaxBlocks = 4096;      // CTAs of a tensor-parallel projection at most
constexpr unsigned kTpStepWord = 16;    // u32 index of the step counter in the header
constexpr unsigned kTpTicketWord = 17;  // u32 index of the exit ticket
constexpr size_t kTpRecvOff = kXchgFlagBytes;
__host__ __device__ constexpr size_t tp_region_bytes(int members, int dim) {
  return kTpRecvOff + 2ull * members * dim * 8;
}

}  // namespace l3p
