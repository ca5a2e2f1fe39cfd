// Constants and the per-step result word shared by every device kernel of
// libl3g and by the host runtime (included inside namespace l3g).
#pragma once

constexpr int NW = 8;                   // consumer warps
constexpr int NTHREADS = 32 * (NW + 1); // + one producer warp
constexpr int MAX_STAGES = 16;
// Shared memory per CTA kept under half an SM's 228 KB, so the next kernel's
// CTA (programmatic dependent launch) can be resident and prefetching.
constexpr int CTA_SMEM_SHARE = 112 * 1024;
// Weight tile target: a 1-D bulk copy costs about 0.25 us per copy per CTA
// on top of its bytes, so copies of ~32 KB are needed to approach HBM speed.
constexpr int TILE_TARGET = 32 * 1024;
constexpr int MAXG = 8;                 // max query heads per kv head
constexpr unsigned long long WAIT_TIMEOUT_NS = 2000000000ull;  // 2 s
constexpr int MAX_TOPK = 64;  // largest top-K a workspace serves
// Waits of a tensor-parallel step: a wait can depend, directly or through the
// kernels launched early behind it, on another GPU's progress, which host
// skew between the ranks' processes can delay by more than the local bound.
constexpr unsigned long long WAIT_TIMEOUT_PEER_NS = 30000000000ull;  // 30 s

// device error codes (Result::err); Result::where names the wait site
enum { ERR_NONE = 0, ERR_TIMEOUT = 1, ERR_TOKEN = 2 };

struct Result {        // copied to the host at the end of every step
  int32_t token;       // argmax id (greedy)
  float logit;         // its logit
  int32_t err;         // ERR_*
  int32_t where;       // wait site / detail
};

// The KV cache in pages.  A page holds KV_PAGE consecutive positions of one
// (layer, local kv head): [KV_PAGE][K hd | V hd] rows of row_bytes each.  A
// state's page table maps (layer, kv head, position / KV_PAGE) to a page of
// a pool: entry (layer * hkv + kv head) * pps + position / KV_PAGE, pps =
// pages per (layer, kv head) for the state's context.  A state with a pool
// of its own maps page j of (layer, kv head) to page (layer * hkv + kv head)
// * pps + j, which is the contiguous layout [layer][kv head][pps *
// KV_PAGE][K | V]; a state in a shared pool takes pages as its position
// grows.  Every bulk copy of K|V rows stays inside one page: copies start at
// multiples of their stage size, which divides KV_PAGE.
constexpr int KV_PAGE = 256;
struct KvMap {
  uint8_t* pool;      // page 0 of the pool
  const int* pages;   // the state's page table (device)
  int pps;            // pages per (layer, kv head)
  int hkv;            // local kv heads
  int row_bytes;      // 2 * head_dim * element bytes
  int pad;
};
__host__ __device__ __forceinline__ size_t kv_page_byte(const KvMap& m, int page, int pos) {
  return ((size_t)page * KV_PAGE + (pos & (KV_PAGE - 1))) * (size_t)m.row_bytes;
}
// The K|V row of (layer, kv head, pos): K at +0, V at + head_dim elements.
__device__ __forceinline__ uint8_t* kv_row(const KvMap& m, int layer, int kvh, int pos) {
  const int page = m.pages[((size_t)layer * m.hkv + kvh) * m.pps + (pos / KV_PAGE)];
  return m.pool + kv_page_byte(m, page, pos);
}

// Dynamic shared memory of a kernel (one declaration per kernel body).  A
// host-side build of the kernels for their CPU checks supplies its own
// definition before including this file.
#ifndef L3G_DYNAMIC_SMEM
#define L3G_DYNAMIC_SMEM(name) extern __shared__ __align__(1024) uint8_t name[]
#endif
