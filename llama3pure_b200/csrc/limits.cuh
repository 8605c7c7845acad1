// limits.cuh -- sizes shared by the NVLink group kernels (seq_xchg.cuh, wo.cuh)
// and the host context (ctx.h).
#pragma once

namespace l3p {

constexpr int kXchgMaxParts = 16;    // members of a sequence or tensor-parallel group
constexpr int kXchgFlagBytes = 256;  // flags and step counter ahead of an exchange region's slots

}  // namespace l3p
