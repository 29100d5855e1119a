// Host-side check: the tcgen05 descriptor encoders of plastic_infer_b200/csrc/umma_desc.cuh
// against CUTLASS's cute::UMMA::SmemDescriptor / InstrDescriptor bitfields, field by field
// over a grid of addresses, offsets, layouts, shapes and majors. Prints "ok" and exits 0
// when every encoding is identical.
#include <cstdio>
#include <cute/arch/mma_sm100_desc.hpp>
#include "umma_desc.cuh"
int main() {
  int bad = 0, n = 0;
  const uint32_t addrs[] = {0u, 1024u, 0x12340u, 0x3FFF0u, 227u * 1024u};
  const uint32_t offs[] = {16u, 1024u, 2048u, 16384u, 65520u};
  const uint32_t lays[] = {0u, 1u, 2u, 4u, 6u};
  for (uint32_t a : addrs) for (uint32_t l : offs) for (uint32_t s : offs) for (uint32_t t : lays)
    for (uint32_t b = 0; b < 8; ++b) {
      cute::UMMA::SmemDescriptor d;
      d.start_address_ = static_cast<uint16_t>(a >> 4);
      d.leading_byte_offset_ = static_cast<uint16_t>(l >> 4);
      d.stride_byte_offset_ = static_cast<uint16_t>(s >> 4);
      d.version_ = 1;
      d.base_offset_ = b;
      d.lbo_mode_ = 0;
      d.layout_type_ = static_cast<uint8_t>(t);
      const uint64_t mine = pi::umma::smem_desc(a, l, s, t, b);
      ++n;
      if (static_cast<uint64_t>(d) != mine) {
        if (bad++ < 5) printf("smem mismatch a=%u l=%u s=%u t=%u b=%u: %016llx vs %016llx\n", a, l, s, t, b,
                              (unsigned long long)(uint64_t)d, (unsigned long long)mine);
      }
    }
  const int ms[] = {64, 128, 256};
  for (int bf = 0; bf < 2; ++bf) for (int m : ms) for (int nn = 8; nn <= 256; nn += 8)
    for (int am = 0; am < 2; ++am) for (int bm = 0; bm < 2; ++bm) {
      cute::UMMA::InstrDescriptor d;
      d.desc_ = 0;
      d.c_format_ = 1;
      d.a_format_ = bf;
      d.b_format_ = bf;
      d.a_major_ = am;
      d.b_major_ = bm;
      d.n_dim_ = nn >> 3;
      d.m_dim_ = m >> 4;
      const uint32_t mine = pi::umma::instr_desc_f16(bf != 0, m, nn, am != 0, bm != 0);
      ++n;
      if (static_cast<uint32_t>(d) != mine) {
        if (bad++ < 10) printf("instr mismatch bf=%d m=%d n=%d am=%d bm=%d: %08x vs %08x\n", bf, m, nn, am, bm,
                               (uint32_t)d, mine);
      }
    }
  printf("%s %d cases, %d mismatches\n", bad ? "FAIL" : "ok", n, bad);
  return bad != 0;
}
