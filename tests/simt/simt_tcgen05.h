// Software versions of the tensor-core helpers of the device code
// (llama3.go_b200/csrc/l3g_tcgen05.cuh), same names and signatures, for the
// host build under the SIMT emulator (simt.h): this file models the
// hardware (namespace simt); simt_tcgen05_helpers.h, included inside
// namespace l3g in place of l3g_tcgen05.cuh, is the helpers.  Test
// infrastructure only.
//
// Modelled after the PTX ISA's description of tcgen05 for cta_group::1:
//   - tensor memory is 128 lanes x 512 columns of 32 bits per CTA, allocated
//     by one warp in power-of-two column ranges of at least 32; the address
//     is lane << 16 | column;
//   - tcgen05.mma kind::i8 with M = 128 writes D[m][n] (lane m, column n
//     from the destination address) = A[m][:] . B[n][:] over K = 32 int8,
//     plus D when accumulating; A (M x K) and B (N x K) are K-major,
//     no-swizzle canonical layouts in shared memory: element (row, k) at
//     start + (row / 8) * SBO + (k / 16) * LBO + (row % 8) * 16 + k % 16,
//     from the descriptors' start address, leading byte offset (LBO) and
//     stride byte offset (SBO); the instruction descriptor gives M, N, the
//     operand and accumulator types;
//   - an MMA runs asynchronously: it reads its operands at some later time,
//     in issue order with the issuing thread's other tensor-core operations,
//     and tcgen05.commit arrives once on an mbarrier when every operation
//     the thread issued before it has completed;
//   - tcgen05.ld.32x32b: lane i of warp w reads tensor-memory lane
//     32 * (w % 4) + i; a warp may only address its own quarter of lanes.
#pragma once

namespace simt {

inline void tmem_cells(Block* b) {
  if (b->tmem.empty()) b->tmem.assign(128 * 512, 0xDEADBEEFu);
}

inline void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  Block* b = cur()->blk;
  if (ncols < 32 || ncols > 512 || (ncols & (ncols - 1)))
    fail("tcgen05.alloc: columns not a power of two in [32, 512]");
  if (b->tmem_relinquished) fail("tcgen05.alloc after relinquish_alloc_permit");
  if (!in_smem(b, dst, 4)) fail("tcgen05.alloc: destination outside shared memory");
  tmem_cells(b);
  const uint32_t units = ncols / 32;
  for (uint32_t u0 = 0; u0 + units <= 16; u0 += units) {
    const uint32_t mask = ((units == 16) ? 0xFFFFu : ((1u << units) - 1u)) << u0;
    if (!(b->tmem_used & mask)) {
      b->tmem_used |= mask;
      *dst = u0 * 32;  // lane 0, first column
      return;
    }
  }
  fail("tcgen05.alloc: no free tensor memory");
}

inline void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  Block* b = cur()->blk;
  const uint32_t col = taddr & 0xFFFFu, units = ncols / 32;
  if ((taddr >> 16) != 0 || col % 32) fail("tcgen05.dealloc: bad address");
  const uint32_t mask = ((units == 16) ? 0xFFFFu : ((1u << units) - 1u)) << (col / 32);
  if ((b->tmem_used & mask) != mask) fail("tcgen05.dealloc of columns not allocated");
  b->tmem_used &= ~mask;
}

struct SmemDesc {
  uint32_t start, lbo, sbo;
};
inline SmemDesc decode_desc(uint64_t d) {
  if (((d >> 46) & 3u) != 1u) fail("tcgen05 matrix descriptor: version field is not 1");
  if ((d >> 61) & 7u) fail("tcgen05 matrix descriptor: only the no-swizzle layout is modelled");
  if ((d >> 49) & 7u) fail("tcgen05 matrix descriptor: base offset not modelled");
  if ((d >> 52) & 1u) fail("tcgen05 matrix descriptor: absolute leading offset mode not modelled");
  return SmemDesc{(uint32_t)(d & 0x3FFFu) << 4, (uint32_t)((d >> 16) & 0x3FFFu) << 4,
                  (uint32_t)((d >> 32) & 0x3FFFu) << 4};
}

inline void execute_mma(const TensorOp& op) {
  Block* b = op.blk;
  const uint32_t idesc = op.idesc;
  if (((idesc >> 4) & 3u) != 2u) fail("tcgen05.mma kind::i8: accumulator type is not s32");
  const uint32_t at = (idesc >> 7) & 7u, bt = (idesc >> 10) & 7u;
  if (at > 1 || bt > 1) fail("tcgen05.mma kind::i8: operand type is neither u8 nor s8");
  if ((idesc >> 15) & 3u) fail("tcgen05.mma: only K-major operands are modelled");
  const int M = (int)((idesc >> 24) & 0x1Fu) << 4, N = (int)((idesc >> 17) & 0x3Fu) << 3;
  if (M != 128) fail("tcgen05.mma cta_group::1: only M = 128 is modelled");
  if (N < 16 || N > 256 || N % 16) fail("tcgen05.mma: N must be a multiple of 16 in [16, 256]");
  const SmemDesc A = decode_desc(op.adesc), B = decode_desc(op.bdesc);
  const uint32_t lane0 = op.d_tmem >> 16, col0 = op.d_tmem & 0xFFFFu;
  if (lane0 != 0) fail("tcgen05.mma: M = 128 needs the accumulator at lane 0");
  for (uint32_t u = col0 / 32; u <= (col0 + N - 1) / 32; ++u)
    if (!(b->tmem_used >> u & 1u)) fail("tcgen05.mma writes tensor memory that is not allocated");
  auto at_byte = [&](const SmemDesc& d, int row, int k) -> const uint8_t* {
    const size_t off = d.start + (size_t)(row / 8) * d.sbo + (size_t)(k / 16) * d.lbo +
                       (size_t)(row % 8) * 16 + (size_t)(k % 16);
    if (off >= b->smem_bytes) fail("tcgen05.mma operand outside shared memory");
    return b->smem + off;
  };
  auto val = [](const uint8_t* p, bool sgn) { return sgn ? (int)(int8_t)*p : (int)*p; };
  for (int m = 0; m < M; ++m) {
    for (int n = 0; n < N; ++n) {
      int acc = 0;
      for (int k = 0; k < 32; ++k)
        acc += val(at_byte(A, m, k), at == 1) * val(at_byte(B, n, k), bt == 1);
      uint32_t& cell = b->tmem[(size_t)(lane0 + m) * 512 + col0 + n];
      cell = (uint32_t)(op.accumulate ? (int)cell + acc : acc);
    }
  }
}

inline void queue_tensor_op(TensorOp op) {
  Runtime& r = rt();
  op.blk = cur()->blk;
  op.issuer = cur();
  const int d = r.randomize ? (int)(r.rng() % (uint64_t)(r.max_copy_delay + 1)) : 1;
  op.due = r.clock + 1 + (uint64_t)d * (r.threads.size() / 8 + 1);
  r.tensor_ops.push_back(op);
}

}  // namespace simt
