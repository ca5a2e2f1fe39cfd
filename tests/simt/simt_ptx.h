// Software versions of the inline-PTX helpers of the device code
// (llama3.go_b200/csrc/l3g_ptx.cuh), same names and signatures, for the
// host build of the kernels under the SIMT emulator (simt.h).  Included
// inside namespace l3g in place of l3g_ptx.cuh.  Test infrastructure only.
#pragma once

inline uint32_t smem_u32(const void* p) {
  return (uint32_t)((const uint8_t*)p - ::simt::dyn_smem());
}
inline void mbar_init(uint64_t* b, uint32_t count) { ::simt::mbar_init(b, count); }
inline void fence_mbar_init() {}
inline void mbar_arrive_expect_tx(uint64_t* b, uint32_t bytes) {
  ::simt::mbar_expect_tx(b, bytes);
  ::simt::mbar_arrive(b);
}
inline void mbar_arrive(uint64_t* b) { ::simt::mbar_arrive(b); }
inline bool mbar_test(uint64_t* b, uint32_t parity) { return ::simt::mbar_test(b, parity); }
inline void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  ::simt::bulk_copy(dst, src, bytes, bar);
}
// Launches run one at a time to completion, so the dependency wait is met
// on entry and the early launch of dependents is a no-op.
inline void pdl_launch_dependents() {}
inline void pdl_wait() {}
inline void touch_page(const void*) {}
inline unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) { return atomicAdd(p, v); }
inline void red_release_gpu_add(unsigned* p, unsigned v) { atomicAdd(p, v); }
inline unsigned atom_add_acq_rel_cta_shared(unsigned* p, unsigned v) { return atomicAdd(p, v); }
inline unsigned ld_acquire_gpu_u32(const unsigned* p) {
  ::simt::cur()->wait = "ld.acquire.gpu (spin)";
  ::simt::yield();
  return *(const volatile unsigned*)p;
}
inline unsigned ld_acquire_sys_u32(const unsigned* p) {
  ::simt::cur()->wait = "ld.acquire.sys (spin)";
  ::simt::yield();
  return *(const volatile unsigned*)p;
}
inline void st_release_sys_u32(unsigned* p, unsigned v) { *(volatile unsigned*)p = v; }
inline unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  ::simt::cur()->wait = "ld.relaxed.sys (spin)";
  ::simt::yield();
  return *(const volatile unsigned long long*)p;
}
inline void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  *(volatile unsigned long long*)p = v;
}
inline uint32_t cluster_ctarank() { ::simt::fail("thread-block clusters are not emulated"); }
inline void cluster_sync_all() { ::simt::fail("thread-block clusters are not emulated"); }
inline float ld_cluster_f32(const float*, uint32_t) {
  ::simt::fail("thread-block clusters are not emulated");
}
inline void consumer_sync() { ::simt::bar_sync(1, NW * 32); }
inline uint64_t gtime() {
  ::simt::yield();
  return ::simt::now();
}
inline void fence_proxy_async_global() {}
