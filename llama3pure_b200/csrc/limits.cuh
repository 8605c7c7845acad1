// limits.cuh -- sizes shared by the NVLink group kernels (seq_xchg.cuh, wo.cuh)
// and the host context (ctx.h).
#pragma once
#include <cstddef>

namespace l3p {

constexpr int kXchgMaxParts = 16;    // members of a sequence or tensor-parallel group
constexpr int kXchgFlagBytes = 256;  // flags and step counter ahead of an exchange region's slots

// Exchange region of a tensor-parallel group (wo.cuh), byte offsets:
//   [0, 256)        header: u32 step (calls completed) at 64, u32 exit ticket at 68
//   kTpArrOff       u32 arrivals[kTpMaxBlocks]: member contributions to row block j
//                   (counted on the block's owner, member j % n_members)
//   kTpDoneOff      u32 done[kTpMaxBlocks]: summed row blocks received, per block
//   kTpRecvOff      float recv[2][n_members][dim]: partial rows sent to this owner
//   tp_result_off   float result[2][dim]: summed rows broadcast by the owners
// Counters only grow (call e expects arrivals e * n_members and done e); the
// slots alternate by call parity.
constexpr int kTpMaxBlocks = 4096;
constexpr unsigned kTpStepWord = 16;    // u32 index of the step counter in the header
constexpr unsigned kTpTicketWord = 17;  // u32 index of the exit ticket
constexpr size_t kTpArrOff = kXchgFlagBytes;
constexpr size_t kTpDoneOff = kTpArrOff + 4ull * kTpMaxBlocks;
constexpr size_t kTpRecvOff = kTpDoneOff + 4ull * kTpMaxBlocks;
__host__ __device__ constexpr size_t tp_result_off(int members, int dim) {
  return kTpRecvOff + 2ull * members * dim * sizeof(float);
}
__host__ __device__ constexpr size_t tp_region_bytes(int members, int dim) {
  return tp_result_off(members, dim) + 2ull * dim * sizeof(float);
}

}  // namespace l3p
