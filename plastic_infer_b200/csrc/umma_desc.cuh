// Encoders of the two descriptors a tcgen05.mma (UMMA) instruction takes, for sm_100a.
//
// Field layout as PTX documents it for tcgen05 (and as CUTLASS's cute::UMMA::SmemDescriptor
// and cute::UMMA::InstrDescriptor bitfields spell it; tests/test_umma_desc.py checks these
// encoders against those unions bit for bit on the host).
//
// Shared-memory matrix descriptor, 64 bits:
//   [ 0,14) start address >> 4        [16,30) leading byte offset >> 4
//   [32,46) stride byte offset >> 4   [46,48) version (1 on sm_100)
//   [49,52) base offset               [52,53) leading-offset mode (0: legacy)
//   [61,64) layout: 0 none, 1 128B with 32B base, 2 128B, 4 64B, 6 32B swizzle
// Canonical tiles with the 128-byte swizzle (element size e, T = 16 / e elements):
//   K-major : rows of the M (or N) dimension 128 bytes apart, 8-row groups `sbo` bytes
//             apart (1024 for a dense tile); one instruction reads a 16-byte-aligned K slice
//             of 2T elements, and the next K slice starts 32 bytes further on.
//   MN-major: 64-element (128-byte) runs along M (or N), `lbo` bytes between runs; K rows
//             128 bytes apart in groups of 8, `sbo` bytes between groups.
//
// Instruction descriptor for kind::f16 (dense), 32 bits:
//   [ 4, 6) D format (1: f32)        [ 7,10) A format (0: f16, 1: bf16)
//   [10,13) B format                 [13,15) negate A / B
//   [15,16) A major (0: K, 1: MN)    [16,17) B major
//   [17,23) N >> 3                   [24,29) M >> 4
#pragma once

#include <cstdint>

namespace pi {
namespace umma {

enum Layout : uint32_t {
  kSwizzleNone = 0,
  kSwizzle128Base32 = 1,
  kSwizzle128 = 2,
  kSwizzle64 = 4,
  kSwizzle32 = 6,
};

__host__ __device__ constexpr uint64_t smem_desc(uint32_t smem_addr, uint32_t lbo_bytes,
                                                 uint32_t sbo_bytes, uint32_t layout,
                                                 uint32_t base_offset = 0) {
  return static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) |
         (static_cast<uint64_t>(1) << 46) |  // version
         (static_cast<uint64_t>(base_offset & 7u) << 49) |
         (static_cast<uint64_t>(layout & 7u) << 61);
}

// kind::f16 with an f32 accumulator: A and B both bf16 (bf16 = true) or both f16.
__host__ __device__ constexpr uint32_t instr_desc_f16(bool bf16, int m, int n, bool a_mn_major,
                                                      bool b_mn_major) {
  return (1u << 4) |                                        // D: f32
         ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |  // A, B format
         ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((static_cast<uint32_t>(n) >> 3) << 17) | ((static_cast<uint32_t>(m) >> 4) << 24);
}

}  // namespace umma
}  // namespace pi
