// Host-only check of the batched product's tcgen05 encodings against the
// CUTLASS sm100 definitions (built and run by tests/test_gemm_layout.py; no
// GPU needed).
//  1. the kind::i8 instruction descriptor for every token tile equals
//     cute::UMMA::make_instr_desc<int8, int8, int32, 128, N, K, K>;
//  2. the shared-memory descriptors of the weight and activation chunks equal
//     cute::UMMA::make_umma_desc<K> of the same canonical layouts (CUTLASS
//     also checks that the layouts are canonical K-major ones); on the host
//     CUTLASS cannot turn a shared-memory pointer into an address, so the
//     start address field is compared on its own;
//  3. prints the descriptors of every block of a chunk staged at fixed
//     addresses, for the test's replay of what the MMA reads.
#include <cstdio>

#include <cute/atom/mma_traits_sm100.hpp>
#include <cute/tensor.hpp>

#include "l3g_gemm_layout.h"

using namespace cute;
namespace G = l3g::gemm;

static int bad = 0;

template <int NT>
static void check_instr() {
  const uint32_t c = (uint32_t)UMMA::make_instr_desc<int8_t, int8_t, int32_t, 128, NT,
                                                     UMMA::Major::K, UMMA::Major::K>();
  const uint32_t o = G::idesc_i8(128, NT);
  std::printf("idesc %d %08x %08x\n", NT, c, o);
  if (c != o) ++bad;
}

template <int NT>
static void check_smem() {
  // weight chunk, block 0: rows (m%8)*16 + (m/8)*128, columns (k%16) + (k/16)*SLAB_A
  auto la = Layout<Shape<Shape<_8, _16>, Shape<_16, _2>>,
                   Stride<Stride<_16, _128>, Stride<_1, Int<G::SLAB_A>>>>{};
  auto ta = make_tensor(make_smem_ptr(reinterpret_cast<int8_t*>(uintptr_t(0x400))), la);
  const uint64_t ca = UMMA::make_umma_desc<UMMA::Major::K>(ta).desc_;
  // activation chunk, block 0: tokens (n%8)*16 + (n/8)*128, columns (k%16) + (k/16)*NT*16
  auto lb = Layout<Shape<Shape<_8, Int<NT / 8>>, Shape<_16, _2>>,
                   Stride<Stride<_16, _128>, Stride<_1, Int<NT * 16>>>>{};
  auto tb = make_tensor(make_smem_ptr(reinterpret_cast<int8_t*>(uintptr_t(0x400))), lb);
  const uint64_t cb = UMMA::make_umma_desc<UMMA::Major::K>(tb).desc_;
  const uint64_t mask = ~0x3FFFull;  // all but the start address
  const uint64_t oa = G::a_desc(0x400, 0), ob = G::b_desc(0x400, 0, NT);
  std::printf("sdesc %d %016llx %016llx %016llx %016llx\n", NT, (unsigned long long)ca,
              (unsigned long long)oa, (unsigned long long)cb, (unsigned long long)ob);
  if ((ca & mask) != (oa & mask) || (cb & mask) != (ob & mask)) ++bad;
  if ((oa & 0x3FFF) != (0x400 >> 4) || (ob & 0x3FFF) != (0x400 >> 4)) ++bad;
}

template <int NT>
static void print_blocks(uint32_t a0) {
  const uint32_t b0 = a0 + G::A_CHUNK;
  for (int j = 0; j < G::BPC; ++j)
    std::printf("block %d %d %u %u %016llx %016llx\n", NT, j, a0, b0,
                (unsigned long long)G::a_desc(a0, j), (unsigned long long)G::b_desc(b0, j, NT));
}

int main() {
  check_instr<16>();
  check_instr<32>();
  check_instr<64>();
  check_instr<128>();
  check_smem<16>();
  check_smem<32>();
  check_smem<64>();
  check_smem<128>();
  const uint32_t a0 = G::SMEM_HEAD + 3 * G::stage_bytes(64);  // a stage in the ring
  print_blocks<16>(G::SMEM_HEAD);
  print_blocks<32>(G::SMEM_HEAD);
  print_blocks<64>(a0);
  print_blocks<128>(G::SMEM_HEAD);
  std::printf("result %d\n", bad);
  return bad ? 1 : 0;
}
