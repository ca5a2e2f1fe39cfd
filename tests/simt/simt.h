// A cooperative SIMT emulator for running the library's device code on the
// host in the CPU test suite (no GPU).  Test infrastructure only.
//
// Every CUDA thread of a launch is a coroutine (ucontext) with its own stack;
// one OS thread schedules them.  A coroutine runs until it reaches a point
// where real hardware could interleave it with other threads -- a warp
// collective, a CTA barrier, an mbarrier poll, an acquire load, an atomic,
// the global timer -- and yields there.  The primitives have the CUDA / PTX
// semantics the kernels rely on:
//   - warp collectives (__shfl*_sync, __all_sync, __syncwarp) exchange values
//     once every lane of the mask has arrived, and fail on an exited lane;
//   - named CTA barriers (bar.sync id, count) release after `count` arrivals;
//   - mbarriers keep a pending-arrival count, a transaction-byte count and a
//     phase; try_wait.parity P is true once the phase of parity P completed;
//   - 1-D bulk copies read their source when issued and land in shared
//     memory after a random delay, then complete their bytes on the mbarrier
//     (so a copy issued before its data was written delivers stale bytes);
//   - shared memory starts filled with 0xCD and ends on a guard page, and
//     global buffers from simt::dmalloc end on a guard page, so reads of
//     uninitialised shared memory show up as garbage and overruns fault;
//   - the schedule is round-robin or, with a seed, a random permutation per
//     round; a run where no thread makes progress for many rounds is
//     reported as a deadlock with every thread's wait site.
// Memory is sequentially consistent (one OS thread), so the emulator checks
// schedules, indexing and barrier logic, not the hardware memory model.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <sys/mman.h>
#include <ucontext.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

namespace simt {

struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};

[[noreturn]] inline void fail(const std::string& msg) { throw Error(msg); }

struct Block;

struct Thread {
  ucontext_t ctx;
  void* stack = nullptr;
  size_t stack_bytes = 0;
  uint3 tid{};
  int linear = 0, lane = 0, warp = 0;
  Block* blk = nullptr;
  bool started = false, done = false;
  const char* wait = "";  // the primitive the thread waits in (diagnostics)
};

struct WarpColl {
  int arrived = 0, departed = 0, expected = 0;
  bool draining = false;
  uint64_t vals[32];
  uint32_t mask = 0;
};

struct Bar {
  int arrived = 0;
  uint64_t gen = 0;
};

struct Block {
  uint3 bidx{};
  uint8_t* smem = nullptr;  // dynamic shared memory (ends on a guard page)
  size_t smem_bytes = 0;
  void* map = nullptr;
  size_t map_bytes = 0;
  std::vector<Thread*> threads;
  std::vector<WarpColl> warps;
  Bar bars[16];
  // tensor memory: 128 lanes x 512 columns of 32 bits, allocated in
  // power-of-two column ranges of at least 32
  std::vector<uint32_t> tmem;
  uint32_t tmem_used = 0;  // bit i: columns [32i, 32i + 32) allocated
  bool tmem_relinquished = false;
};

// An asynchronous tensor-core operation (tcgen05.mma or tcgen05.commit),
// executed in issue order per issuing thread after a delay.
struct TensorOp {
  bool commit;
  Block* blk;
  Thread* issuer;
  uint64_t due;
  uint32_t d_tmem;
  uint64_t adesc, bdesc;
  uint32_t idesc, accumulate;
  uint64_t* bar;
};

struct MBar {
  uint32_t count = 0, pending = 0;
  int64_t tx = 0;
  uint64_t phase = 0;  // completed phases
};

struct Copy {
  uint8_t* dst;
  std::vector<uint8_t> data;
  uint64_t* bar;
  Block* blk;
  uint64_t due;
};

struct Alloc {
  void* map;
  size_t map_bytes;
  size_t bytes;
};

struct Runtime {
  ucontext_t sched;
  Thread* cur = nullptr;
  std::vector<Thread*> threads;
  std::vector<Block*> blocks;
  dim3 grid, block;
  uint64_t clock = 0;      // fake %globaltimer, ns
  uint64_t progress = 0;   // bumped whenever some thread gets past a wait
  std::vector<Copy> copies;
  std::vector<TensorOp> tensor_ops;
  std::map<uint64_t*, MBar> mbars;
  std::map<uintptr_t, Alloc> allocs;  // base -> allocation
  std::mt19937_64 rng{1};
  bool randomize = false;
  int max_copy_delay = 64;
  std::function<void()> body;
  std::string error;
};

inline Runtime& rt() {
  static Runtime r;
  return r;
}
inline Thread* cur() { return rt().cur; }

inline size_t page() { return (size_t)sysconf(_SC_PAGESIZE); }

// block index and grid size seen by the kernel in a sequential launch
inline bool& seq_override() {
  static bool v = false;
  return v;
}
inline uint3& seq_bidx() {
  static uint3 v{};
  return v;
}
inline dim3& seq_grid() {
  static dim3 v;
  return v;
}

// ---------------------------------------------------------------------------
// memory
// ---------------------------------------------------------------------------
// `bytes` of zeroed memory whose end abuts a PROT_NONE page; the start is
// 256-byte aligned (bytes are rounded up to 256).
inline void* guarded(size_t bytes, void** map_out, size_t* map_bytes_out) {
  const size_t pg = page();
  const size_t body = (bytes + 255) / 256 * 256;
  const size_t span = (body + pg - 1) / pg * pg + pg;
  void* m = mmap(nullptr, span, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
  if (m == MAP_FAILED) fail("mmap failed");
  uint8_t* guard = static_cast<uint8_t*>(m) + span - pg;
  if (mprotect(guard, pg, PROT_NONE) != 0) fail("mprotect failed");
  *map_out = m;
  *map_bytes_out = span;
  return guard - body;
}

// A device buffer: zeroed, 256-byte aligned, ends on a guard page.
inline void* dmalloc(size_t bytes) {
  void* m;
  size_t mb;
  void* p = guarded(bytes ? bytes : 1, &m, &mb);
  rt().allocs[(uintptr_t)p] = Alloc{m, mb, bytes};
  return p;
}
inline void dfree(void* p) {
  auto it = rt().allocs.find((uintptr_t)p);
  if (it == rt().allocs.end()) fail("dfree of an unknown pointer");
  munmap(it->second.map, it->second.map_bytes);
  rt().allocs.erase(it);
}
// Whether [p, p + n) lies inside one dmalloc buffer.
inline bool in_global(const void* p, size_t n) {
  auto& a = rt().allocs;
  auto it = a.upper_bound((uintptr_t)p);
  if (it == a.begin()) return false;
  --it;
  return (uintptr_t)p + n <= it->first + it->second.bytes;
}
inline bool in_smem(const Block* b, const void* p, size_t n) {
  return (const uint8_t*)p >= b->smem && (const uint8_t*)p + n <= b->smem + b->smem_bytes;
}

// ---------------------------------------------------------------------------
// scheduling
// ---------------------------------------------------------------------------
inline void yield() {
  Thread* t = cur();
  swapcontext(&t->ctx, &rt().sched);
}
inline void made_progress() { ++rt().progress; }

inline void deliver_copies(bool all) {
  Runtime& r = rt();
  for (size_t i = 0; i < r.copies.size();) {
    if (all || r.copies[i].due <= r.clock) {
      Copy c = std::move(r.copies[i]);
      r.copies.erase(r.copies.begin() + i);
      memcpy(c.dst, c.data.data(), c.data.size());
      auto it = r.mbars.find(c.bar);
      if (it == r.mbars.end()) fail("bulk copy completes on an uninitialised mbarrier");
      MBar& m = it->second;
      m.tx -= (int64_t)c.data.size();
      if (m.pending == 0 && m.tx == 0) {
        ++m.phase;
        m.pending = m.count;
      }
      made_progress();
    } else {
      ++i;
    }
  }
}

inline void execute_mma(const TensorOp& op);  // simt_tcgen05.h

inline void deliver_tensor_ops(bool all) {
  Runtime& r = rt();
  std::vector<Thread*> blocked;
  for (size_t i = 0; i < r.tensor_ops.size();) {
    TensorOp& op = r.tensor_ops[i];
    const bool waits = std::find(blocked.begin(), blocked.end(), op.issuer) != blocked.end();
    if (!waits && (all || op.due <= r.clock)) {
      const TensorOp o = op;
      r.tensor_ops.erase(r.tensor_ops.begin() + i);
      if (o.commit) {
        auto it = r.mbars.find(o.bar);
        if (it == r.mbars.end()) fail("tcgen05.commit to an uninitialised mbarrier");
        MBar& m = it->second;
        if (m.pending == 0) fail("tcgen05.commit arrives on a completed phase");
        --m.pending;
        if (m.pending == 0 && m.tx == 0) {
          ++m.phase;
          m.pending = m.count;
        }
      } else {
        execute_mma(o);
      }
      made_progress();
    } else {
      blocked.push_back(op.issuer);
      ++i;
    }
  }
}

inline void trampoline() {
  Thread* t = cur();
  try {
    rt().body();
  } catch (const Error& e) {
    if (rt().error.empty()) rt().error = e.what();
  }
  t->done = true;
  made_progress();
  swapcontext(&t->ctx, &rt().sched);
}

// Runs body() as every thread of a grid x block launch with `smem` bytes of
// dynamic shared memory per block, to completion.  Throws simt::Error on a
// deadlock or on a failed check inside the emulated code.
inline void launch(dim3 grid, dim3 block, size_t smem, std::function<void()> body,
                   bool sequential = false, size_t stack_bytes = 256 * 1024);

// With sequential = true the blocks run one after another (each to
// completion), as kernels with static shared arrays need here.
inline void launch(dim3 grid, dim3 block, size_t smem, std::function<void()> body,
                   bool sequential, size_t stack_bytes) {
  if (sequential && grid.x * grid.y * grid.z > 1) {
    const std::function<void()> b = body;
    for (unsigned z = 0; z < grid.z; ++z)
      for (unsigned y = 0; y < grid.y; ++y)
        for (unsigned x = 0; x < grid.x; ++x) {
          // a one-block launch whose block index and grid size read as the
          // full launch's
          launch(dim3(1), block, smem, [&, x, y, z] {
            seq_override() = true;
            seq_bidx() = uint3{x, y, z};
            seq_grid() = grid;
            b();
          });
          seq_override() = false;
        }
    return;
  }
  Runtime& r = rt();
  r.grid = grid;
  r.block = block;
  r.body = std::move(body);
  r.error.clear();
  r.mbars.clear();
  r.copies.clear();
  r.tensor_ops.clear();
  const int nb = (int)(grid.x * grid.y * grid.z);
  const int nt = (int)(block.x * block.y * block.z);
  for (int b = 0; b < nb; ++b) {
    Block* B = new Block;
    B->bidx = uint3{(unsigned)(b % grid.x), (unsigned)((b / grid.x) % grid.y),
                    (unsigned)(b / (grid.x * grid.y))};
    B->smem_bytes = (smem + 1023) / 1024 * 1024;
    if (B->smem_bytes) {
      B->smem = static_cast<uint8_t*>(guarded(B->smem_bytes, &B->map, &B->map_bytes));
      memset(B->smem, 0xCD, B->smem_bytes);
    }
    B->warps.resize((nt + 31) / 32);
    for (int i = 0; i < nt; ++i) {
      Thread* t = new Thread;
      t->tid = uint3{(unsigned)(i % block.x), (unsigned)((i / block.x) % block.y),
                     (unsigned)(i / (block.x * block.y))};
      t->linear = i;
      t->lane = i & 31;
      t->warp = i >> 5;
      t->blk = B;
      t->stack_bytes = stack_bytes;
      t->stack = mmap(nullptr, stack_bytes, PROT_READ | PROT_WRITE,
                      MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE, -1, 0);
      if (t->stack == MAP_FAILED) fail("stack mmap failed");
      B->threads.push_back(t);
      r.threads.push_back(t);
    }
    r.blocks.push_back(B);
  }
  std::vector<Thread*> order = r.threads;
  uint64_t idle_rounds = 0, last_progress = r.progress;
  size_t alive = order.size();
  while (alive) {
    if (r.randomize) std::shuffle(order.begin(), order.end(), r.rng);
    for (Thread* t : order) {
      if (t->done) continue;
      if (!t->started) {
        t->started = true;
        getcontext(&t->ctx);
        t->ctx.uc_stack.ss_sp = t->stack;
        t->ctx.uc_stack.ss_size = t->stack_bytes;
        t->ctx.uc_link = nullptr;
        makecontext(&t->ctx, trampoline, 0);
      }
      r.cur = t;
      swapcontext(&r.sched, &t->ctx);
      r.cur = nullptr;
      ++r.clock;
      if (t->done) --alive;
      if (!r.error.empty()) break;
    }
    try {
      deliver_copies(false);
      deliver_tensor_ops(false);
    } catch (const Error& e) {
      if (r.error.empty()) r.error = e.what();
    }
    if (!r.error.empty()) break;
    if (r.progress != last_progress) {
      last_progress = r.progress;
      idle_rounds = 0;
    } else if (++idle_rounds > 20000) {
      if (!r.copies.empty() || !r.tensor_ops.empty()) {
        try {
          deliver_copies(true);
          deliver_tensor_ops(true);
        } catch (const Error& e) {
          if (r.error.empty()) r.error = e.what();
          break;
        }
        continue;
      }
      std::string msg = "deadlock: no thread progressed; waits:";
      std::map<std::string, int> sites;
      for (Thread* t : r.threads)
        if (!t->done)
          sites[std::string(t->wait) + " (block " + std::to_string(t->blk->bidx.x) + ")"]++;
      for (auto& s : sites) msg += " " + s.first + " x" + std::to_string(s.second) + ";";
      r.error = msg;
      break;
    }
  }
  const std::string err = r.error;
  if (err.empty() && !r.copies.empty()) r.error = "bulk copies still in flight at kernel exit";
  if (r.error.empty() && !r.tensor_ops.empty())
    r.error = "tensor-core operations still in flight at kernel exit";
  for (Block* B : r.blocks)
    if (r.error.empty() && B->tmem_used)
      r.error = "tensor memory still allocated at kernel exit";
  const std::string err2 = r.error;
  for (Thread* t : r.threads) {
    munmap(t->stack, t->stack_bytes);
    delete t;
  }
  for (Block* B : r.blocks) {
    if (B->map) munmap(B->map, B->map_bytes);
    delete B;
  }
  r.threads.clear();
  r.blocks.clear();
  r.copies.clear();
  r.tensor_ops.clear();
  if (!err2.empty()) fail(err2);
}

// ---------------------------------------------------------------------------
// built-in variables
// ---------------------------------------------------------------------------
inline const uint3& thread_idx() { return cur()->tid; }
inline const uint3& block_idx() { return seq_override() ? seq_bidx() : cur()->blk->bidx; }
inline const dim3& block_dim() { return rt().block; }
inline const dim3& grid_dim() { return seq_override() ? seq_grid() : rt().grid; }
inline uint8_t* dyn_smem() { return cur()->blk->smem; }

// ---------------------------------------------------------------------------
// warp collectives
// ---------------------------------------------------------------------------
// Every lane of `mask` deposits v; returns the value deposited by lane
// src(lane) (or the caller's own when src < 0 or >= 32), and through
// *all_vals every lane's value.
inline uint64_t warp_exchange(uint32_t mask, uint64_t v, int src, const char* what,
                              uint64_t* all_vals = nullptr) {
  Thread* t = cur();
  if (!(mask >> t->lane & 1u)) fail(std::string(what) + ": calling lane not in the mask");
  Block* B = t->blk;
  WarpColl& w = B->warps[t->warp];
  t->wait = what;
  while (w.draining) yield();
  if (w.arrived == 0) {
    w.mask = mask;
    w.expected = __builtin_popcount(mask);
  } else if (w.mask != mask) {
    fail(std::string(what) + ": lanes of one warp disagree on the mask");
  }
  for (int l = 0; l < 32; ++l) {
    const int idx = t->warp * 32 + l;
    if ((mask >> l & 1u) && (idx >= (int)B->threads.size() || B->threads[idx]->done))
      fail(std::string(what) + ": a lane of the mask has exited");
  }
  w.vals[t->lane] = v;
  if (++w.arrived == w.expected) {
    w.draining = true;
    made_progress();
  }
  while (!w.draining || w.arrived < w.expected) yield();
  const uint64_t r = (src >= 0 && src < 32 && (mask >> src & 1u)) ? w.vals[src] : v;
  if (all_vals)
    for (int l = 0; l < 32; ++l) all_vals[l] = (mask >> l & 1u) ? w.vals[l] : 0;
  if (++w.departed == w.expected) {
    w.arrived = 0;
    w.departed = 0;
    w.draining = false;
  }
  // let the others read before anyone reuses the slots
  t->wait = "";
  return r;
}

template <typename T>
inline uint64_t to_bits(T v) {
  uint64_t b = 0;
  memcpy(&b, &v, sizeof(T));
  return b;
}
template <typename T>
inline T from_bits(uint64_t b) {
  T v;
  memcpy(&v, &b, sizeof(T));
  return v;
}

// ---------------------------------------------------------------------------
// CTA barriers
// ---------------------------------------------------------------------------
inline void bar_sync(int id, int count) {
  Thread* t = cur();
  Bar& b = t->blk->bars[id];
  const uint64_t gen = b.gen;
  t->wait = id == 0 ? "__syncthreads" : "bar.sync (named)";
  if (++b.arrived == count) {
    b.arrived = 0;
    ++b.gen;
    made_progress();
  } else {
    while (b.gen == gen) yield();
  }
  t->wait = "";
}

// ---------------------------------------------------------------------------
// mbarriers and bulk copies
// ---------------------------------------------------------------------------
inline MBar& mbar(uint64_t* b, const char* what) {
  if (!in_smem(cur()->blk, b, 8) || ((uintptr_t)b & 7))
    fail(std::string(what) + ": mbarrier outside this CTA's shared memory or unaligned");
  auto it = rt().mbars.find(b);
  if (it == rt().mbars.end()) fail(std::string(what) + ": mbarrier not initialised");
  return it->second;
}
inline void mbar_init(uint64_t* b, uint32_t count) {
  if (!in_smem(cur()->blk, b, 8) || ((uintptr_t)b & 7)) fail("mbarrier.init outside shared memory");
  rt().mbars[b] = MBar{count, count, 0, 0};
}
inline void mbar_complete_if_done(MBar& m) {
  if (m.pending == 0 && m.tx == 0) {
    ++m.phase;
    m.pending = m.count;
    made_progress();
  }
}
inline void mbar_arrive(uint64_t* b) {
  MBar& m = mbar(b, "mbarrier.arrive");
  if (m.pending == 0) fail("mbarrier.arrive on a completed phase");
  --m.pending;
  mbar_complete_if_done(m);
}
inline void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  MBar& m = mbar(b, "mbarrier.expect_tx");
  m.tx += bytes;
}
inline bool mbar_test(uint64_t* b, uint32_t parity) {
  cur()->wait = "mbarrier.try_wait";
  yield();
  const MBar& m = mbar(b, "mbarrier.try_wait");
  const bool ok = (m.phase & 1u) != (parity & 1u);
  if (ok) cur()->wait = "";
  return ok;
}
inline void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  Thread* t = cur();
  if (((uintptr_t)dst & 15) || ((uintptr_t)src & 15) || (bytes & 15) || bytes == 0)
    fail("cp.async.bulk: address or size not a multiple of 16 bytes");
  if (!in_smem(t->blk, dst, bytes)) fail("cp.async.bulk: destination outside shared memory");
  if (!in_global(src, bytes)) fail("cp.async.bulk: source outside every device buffer");
  mbar(bar, "cp.async.bulk");
  Runtime& r = rt();
  Copy c;
  c.dst = static_cast<uint8_t*>(dst);
  c.data.assign(static_cast<const uint8_t*>(src), static_cast<const uint8_t*>(src) + bytes);
  c.bar = bar;
  c.blk = t->blk;
  const int d = r.randomize ? (int)(r.rng() % (uint64_t)(r.max_copy_delay + 1)) : 1;
  c.due = r.clock + 1 + (uint64_t)d * (r.threads.size() / 8 + 1);
  r.copies.push_back(std::move(c));
}
inline uint64_t now() { return rt().clock; }

}  // namespace simt

// ---------------------------------------------------------------------------
// CUDA built-ins for the emulated device code
// ---------------------------------------------------------------------------
#undef __global__
#define __global__
#undef __launch_bounds__
#define __launch_bounds__(...)
#undef __grid_constant__
#define __grid_constant__
#define threadIdx (::simt::thread_idx())
#define blockIdx (::simt::block_idx())
#define blockDim (::simt::block_dim())
#define gridDim (::simt::grid_dim())
#define L3G_DYNAMIC_SMEM(name) uint8_t* name = ::simt::dyn_smem()
// Static shared arrays become function statics: one copy for the whole
// launch, so kernels that declare them run with simt::launch(...,
// sequential = true), one block after another.
#undef __shared__
#define __shared__ static

template <typename T>
inline T simt_shfl(uint32_t mask, T v, int src, const char* what) {
  return simt::from_bits<T>(simt::warp_exchange(mask, simt::to_bits(v), src, what));
}
template <typename T>
inline T __shfl_sync(unsigned mask, T v, int src, int width = 32) {
  (void)width;
  return simt_shfl(mask, v, src & 31, "__shfl_sync");
}
template <typename T>
inline T __shfl_xor_sync(unsigned mask, T v, int lm, int width = 32) {
  (void)width;
  return simt_shfl(mask, v, (simt::cur()->lane ^ lm) & 31, "__shfl_xor_sync");
}
template <typename T>
inline T __shfl_down_sync(unsigned mask, T v, unsigned d, int width = 32) {
  (void)width;
  const int s = simt::cur()->lane + (int)d;
  return simt_shfl(mask, v, s < 32 ? s : -1, "__shfl_down_sync");
}
template <typename T>
inline T __shfl_up_sync(unsigned mask, T v, unsigned d, int width = 32) {
  (void)width;
  const int s = simt::cur()->lane - (int)d;
  return simt_shfl(mask, v, s >= 0 ? s : -1, "__shfl_up_sync");
}
inline unsigned __ballot_sync(unsigned mask, int pred) {
  uint64_t all[32];
  simt::warp_exchange(mask, pred ? 1 : 0, -1, "__ballot_sync", all);
  unsigned r = 0;
  for (int l = 0; l < 32; ++l)
    if (all[l]) r |= 1u << l;
  return r;
}
inline int __all_sync(unsigned mask, int pred) { return __ballot_sync(mask, pred) == mask; }
inline int __any_sync(unsigned mask, int pred) { return __ballot_sync(mask, pred) != 0; }
inline void __syncwarp(unsigned mask = 0xffffffffu) {
  simt::warp_exchange(mask, 0, -1, "__syncwarp");
}
inline void __syncthreads() {
  simt::bar_sync(0, (int)(simt::rt().block.x * simt::rt().block.y * simt::rt().block.z));
}
inline void __threadfence() {}
inline void __threadfence_block() {}

// CUDA's integer min / max overloads
inline int min(int a, int b) { return a < b ? a : b; }
inline int max(int a, int b) { return a > b ? a : b; }
inline unsigned min(unsigned a, unsigned b) { return a < b ? a : b; }
inline unsigned max(unsigned a, unsigned b) { return a > b ? a : b; }
inline long long min(long long a, long long b) { return a < b ? a : b; }
inline long long max(long long a, long long b) { return a > b ? a : b; }
inline unsigned long long min(unsigned long long a, unsigned long long b) { return a < b ? a : b; }
inline unsigned long long max(unsigned long long a, unsigned long long b) { return a > b ? a : b; }

// arithmetic with the rounding of the named CUDA intrinsic (the host build
// uses -ffp-contract=off, so a * b + c is never fused behind our back)
inline float __fadd_rn(float a, float b) { return a + b; }
inline float __fsub_rn(float a, float b) { return a - b; }
inline float __fmul_rn(float a, float b) { return a * b; }
inline float __fdiv_rn(float a, float b) { return a / b; }
inline float __frcp_rn(float a) { return 1.0f / a; }
inline int __dp4a(int a, int b, int c) {
  for (int i = 0; i < 4; ++i) c += (int)(int8_t)(a >> (8 * i)) * (int)(int8_t)(b >> (8 * i));
  return c;
}
inline unsigned __float_as_uint(float f) { return simt::from_bits<unsigned>(simt::to_bits(f)); }
inline float __uint_as_float(unsigned u) { return simt::from_bits<float>(simt::to_bits(u)); }
inline int __float_as_int(float f) { return simt::from_bits<int>(simt::to_bits(f)); }
inline float __int_as_float(int u) { return simt::from_bits<float>(simt::to_bits(u)); }
template <typename T>
inline T __ldcg(const T* p) {
  return *p;
}
template <typename T>
inline T __ldg(const T* p) {
  return *p;
}
template <typename T>
inline void __stcg(T* p, T v) {
  *p = v;
}

// atomics: every atomic is a point where another thread may run first
template <typename T>
inline T atomicAdd(T* p, T v) {
  simt::yield();
  const T o = *p;
  *p = o + v;
  simt::made_progress();
  return o;
}
template <typename T>
inline T atomicExch(T* p, T v) {
  simt::yield();
  const T o = *p;
  *p = v;
  simt::made_progress();
  return o;
}
template <typename T>
inline T atomicCAS(T* p, T cmp, T v) {
  simt::yield();
  const T o = *p;
  if (o == cmp) *p = v;
  simt::made_progress();
  return o;
}
