// Data layout of the batched Q8_0 product on the 5th-generation tensor cores
// (tcgen05.mma kind::i8), shared by the device kernels, the host-side repack
// and the layout checks.  Plain C++ (host and device), no CUDA API.
//
// The product is n_tok independent Q8_0 matvecs (matVecQ8_0,
// internal/llama/matvec_cgo.go:14-30 -> matvec_q8_c, simd.c:33-110) over one
// weight matrix, computed as one GEMM: out[n][r] = sum_b d_w[r,b] * d_x[n,b] *
// I_b[r,n], with I_b[r,n] = sum_{i<32} q_w[r,32b+i] * q_x[n,32b+i] exact in
// int32.  One MMA of kind::i8 has K = 32 = one Q8_0 block, so each block's
// integer product lands in tensor memory on its own and the fp32 rescale by
// d_w * d_x happens per block, as in the reference.
//
// Both operands are K-major in the canonical layout without swizzle: 16-byte
// core-matrix rows, 8 rows of a core matrix contiguous (128 bytes).  Within a
// chunk of KC = 128 columns (four Q8_0 blocks) the bytes of row m, column k
// sit at (k / 16) * ROWS * 16 + m * 16 + k % 16: the chunk is 8 slabs of
// 16-byte columns, each slab all rows in order.  So for one MMA (block j,
// columns 32j..32j+31) the descriptor starts at slab 2j, the two K halves of
// a core matrix are one slab apart (leading byte offset = ROWS * 16) and
// consecutive 8-row groups are 128 bytes apart (stride byte offset).
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define L3G_HD __host__ __device__
#else
#define L3G_HD
#endif

namespace l3g {
namespace gemm {

constexpr int TILE_M = 128;   // weight rows per tile = MMA M (TMEM lane = row)
constexpr int KC = 128;       // columns per chunk (one ring stage)
constexpr int QBLK = 32;      // Q8_0 block = K of one kind::i8 MMA
constexpr int BPC = KC / QBLK;  // blocks per chunk
constexpr int SLAB_A = TILE_M * 16;  // bytes of one 16-column slab of a weight chunk

// Weight chunk (row tile rt, chunk c): int8 q [KC/16][TILE_M][16], then the
// fp16 block scales d[BPC][TILE_M].  Chunks are stored rt-major:
// chunk (rt, c) at ((rt * nk) + c) * A_CHUNK.
constexpr int A_Q_BYTES = TILE_M * KC;              // 16384
constexpr int A_D_BYTES = BPC * TILE_M * 2;         // 1024
constexpr int A_CHUNK = A_Q_BYTES + A_D_BYTES;      // 17408
static_assert(A_CHUNK % 128 == 0, "weight chunk alignment");

// Activation chunk (token tile ti of NT tokens, chunk c): int8 q
// [KC/16][NT][16], then the fp32 scales d[BPC][NT]; chunk (ti, c) at
// ((ti * nk) + c) * b_chunk(NT).  Padding tokens (n >= n_tok) are zero.
L3G_HD constexpr int b_q_bytes(int nt) { return nt * KC; }
L3G_HD constexpr int b_chunk(int nt) { return nt * KC + BPC * nt * 4; }

// byte offset of (row m, column k within the chunk) in a chunk of `rows` rows
L3G_HD constexpr int q_offset(int rows, int m, int k) {
  return (k / 16) * rows * 16 + m * 16 + (k % 16);
}

// Token tile of a product over n_tok tokens: the MMA's N (a multiple of 16).
L3G_HD constexpr int token_tile(int n_tok) {
  return n_tok <= 16 ? 16 : n_tok <= 32 ? 32 : n_tok <= 64 ? 64 : 128;
}
L3G_HD constexpr int chunks(int cols) { return (cols + KC - 1) / KC; }
L3G_HD constexpr int row_tiles(int rows) { return (rows + TILE_M - 1) / TILE_M; }

// Shared-memory matrix descriptor (tcgen05 "matrix descriptor"): start
// address, leading and stride byte offsets (all >> 4, 14 bits each), the
// fixed version field of sm_100 (bits 46-47 = 1), base offset 0, leading
// offset mode 0 and layout type 0 (no swizzle, bits 61-63).
L3G_HD constexpr uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Descriptors of block j of a chunk staged at a_base / b_base (shared-memory
// addresses) for a token tile of nt.
L3G_HD constexpr uint64_t a_desc(uint32_t a_base, int j) {
  return smem_desc(a_base + (uint32_t)(2 * j * SLAB_A), SLAB_A, 128);
}
L3G_HD constexpr uint64_t b_desc(uint32_t b_base, int j, int nt) {
  return smem_desc(b_base + (uint32_t)(2 * j * nt * 16), (uint32_t)(nt * 16), 128);
}

// Instruction descriptor of kind::i8: D s32 (bits 4-5 = 2), A and B signed
// int8 (bits 7-9, 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at bits
// 17-22, M >> 4 at bits 24-28; dense, no negation, no saturation.
L3G_HD constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

// CTAs of the product resident per SM: two at 64 tokens, each with half of
// the SM's tensor memory and of its shared-memory ring, so that two CTAs'
// block chains (MMA, commit, tensor-memory load, rescale, release)
// interleave on the SM; one otherwise.
L3G_HD constexpr int ctas_per_sm(int nt) { return nt == 64 ? 2 : 1; }

// Tensor-memory buffers of one CTA: NB buffers of NT columns (one per block
// in flight between the MMA issuer and the rescaling warps), the CTA's share
// of the SM's 512 columns: 32, 16, 4 (two CTAs) and 4 blocks in flight at
// 16, 32, 64 and 128 tokens, so the MMAs run that far ahead of the rescale.
L3G_HD constexpr int tmem_buffers(int nt) {
  return 512 / ctas_per_sm(nt) / nt < 32 ? 512 / ctas_per_sm(nt) / nt : 32;
}
L3G_HD constexpr int tmem_cols(int nt) {
  return tmem_buffers(nt) * nt <= 32 ? 32 : tmem_buffers(nt) * nt <= 64 ? 64
       : tmem_buffers(nt) * nt <= 128 ? 128 : tmem_buffers(nt) * nt <= 256 ? 256 : 512;
}

// Ring stage = one weight chunk + one activation chunk.
L3G_HD constexpr int stage_bytes(int nt) { return A_CHUNK + b_chunk(nt); }
constexpr int SMEM_HEAD = 1024;
constexpr int SMEM_BUDGET = 200 * 1024;     // ring bytes of a CTA alone on its SM
constexpr int SMEM_BUDGET_2 = 107 * 1024;   // each of two CTAs on an SM
constexpr int MAX_STAGES_G = 8;
L3G_HD constexpr int stages(int nt) {
  return ((ctas_per_sm(nt) == 2 ? SMEM_BUDGET_2 : SMEM_BUDGET) / stage_bytes(nt)) < MAX_STAGES_G
             ? ((ctas_per_sm(nt) == 2 ? SMEM_BUDGET_2 : SMEM_BUDGET) / stage_bytes(nt))
             : MAX_STAGES_G;
}
L3G_HD constexpr int smem_bytes(int nt) { return SMEM_HEAD + stages(nt) * stage_bytes(nt); }

}  // namespace gemm
}  // namespace l3g
