// Software versions of the helpers of llama3.go_b200/csrc/l3g_tcgen05.cuh
// (same names and signatures) on the tensor-core model of simt_tcgen05.h.
// Included inside namespace l3g in place of l3g_tcgen05.cuh.  Test
// infrastructure only.
#pragma once


inline void tc_fence_before() {}
inline void tc_fence_after() {}
// whole warp: one allocation of ncols columns, its address to *dst
inline void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  __syncwarp();
  if (::simt::cur()->lane == 0) {
    ::simt::tmem_alloc(dst, ncols);
    ::simt::cur()->blk->tmem_relinquished = true;
  }
  __syncwarp();
}
inline void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  __syncwarp();
  if (::simt::cur()->lane == 0) ::simt::tmem_dealloc(taddr, ncols);
  __syncwarp();
}
inline void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                   uint32_t accumulate) {
  ::simt::TensorOp op{};
  op.commit = false;
  op.d_tmem = d_tmem;
  op.adesc = adesc;
  op.bdesc = bdesc;
  op.idesc = idesc;
  op.accumulate = accumulate;
  ::simt::queue_tensor_op(op);
}
inline void mma_commit(uint64_t* bar) {
  ::simt::mbar(bar, "tcgen05.commit");
  ::simt::TensorOp op{};
  op.commit = true;
  op.bar = bar;
  ::simt::queue_tensor_op(op);
}
// whole warp: lane i reads 8 columns of tensor-memory lane (taddr lane) + i
inline void tmem_ld8(uint32_t taddr, uint32_t* v) {
  ::simt::Thread* t = ::simt::cur();
  __syncwarp();
  const uint32_t lane0 = taddr >> 16, col = taddr & 0xFFFFu;
  if (lane0 != 32u * (uint32_t)(t->warp % 4))
    ::simt::fail("tcgen05.ld: a warp may only read its own quarter of the lanes");
  for (uint32_t u = col / 32; u <= (col + 7) / 32; ++u)
    if (!(t->blk->tmem_used >> u & 1u)) ::simt::fail("tcgen05.ld of unallocated tensor memory");
  for (int i = 0; i < 8; ++i) v[i] = t->blk->tmem[(size_t)(lane0 + t->lane) * 512 + col + i];
}
// whole warp: lane i reads 4 columns of tensor-memory lane (taddr lane) + i
inline void tmem_ld4(uint32_t taddr, uint32_t* v) {
  ::simt::Thread* t = ::simt::cur();
  __syncwarp();
  const uint32_t lane0 = taddr >> 16, col = taddr & 0xFFFFu;
  if (lane0 != 32u * (uint32_t)(t->warp % 4))
    ::simt::fail("tcgen05.ld: a warp may only read its own quarter of the lanes");
  for (uint32_t u = col / 32; u <= (col + 3) / 32; ++u)
    if (!(t->blk->tmem_used >> u & 1u)) ::simt::fail("tcgen05.ld of unallocated tensor memory");
  for (int i = 0; i < 4; ++i) v[i] = t->blk->tmem[(size_t)(lane0 + t->lane) * 512 + col + i];
}
inline void tmem_wait_ld() {}

inline unsigned long long pk2(float a, float b) {
  return (unsigned long long)__float_as_uint(a) | ((unsigned long long)__float_as_uint(b) << 32);
}
inline float2 upk2(unsigned long long r) {
  return make_float2(__uint_as_float((unsigned)r), __uint_as_float((unsigned)(r >> 32)));
}
inline unsigned long long add2(unsigned long long a, unsigned long long b) {
  const float2 x = upk2(a), y = upk2(b);
  return pk2(x.x + y.x, x.y + y.y);
}
inline unsigned long long mul2(unsigned long long a, unsigned long long b) {
  const float2 x = upk2(a), y = upk2(b);
  return pk2(x.x * y.x, x.y * y.y);
}
inline unsigned long long fma2(unsigned long long a, unsigned long long b, unsigned long long c) {
  const float2 x = upk2(a), y = upk2(b), z = upk2(c);
  return pk2(std::fma(x.x, y.x, z.x), std::fma(x.y, y.y, z.y));
}
