// Errors, version, options, the NCCL binding and the failure-detection
// self test of libl3g.
#include "l3g_rt.h"

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------
static thread_local std::string g_err;

int l3g_fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

extern "C" const char* l3g_last_error(void) { return g_err.c_str(); }
extern "C" int l3g_version(void) { return L3G_VERSION; }

extern "C" int l3g_device_count(int32_t* n) {
  int c = 0;
  CUDA_TRY(cudaGetDeviceCount(&c));
  if (n) *n = c;
  return L3G_OK;
}

extern "C" void l3g_options_default(l3g_options* opt) {
  if (!opt) return;
  memset(opt, 0, sizeof *opt);
  opt->world_size = 1;
  opt->rank = 0;
  opt->device = -1;
  opt->kv_dtype = L3G_KV_F32;
}

NcclApi* nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.GetUniqueId = (decltype(api.GetUniqueId))dlsym(h, "ncclGetUniqueId");
    api.CommInitRank = (decltype(api.CommInitRank))dlsym(h, "ncclCommInitRank");
    api.AllReduce = (decltype(api.AllReduce))dlsym(h, "ncclAllReduce");
    api.AllGather = (decltype(api.AllGather))dlsym(h, "ncclAllGather");
    api.CommDestroy = (decltype(api.CommDestroy))dlsym(h, "ncclCommDestroy");
    api.GetErrorString = (decltype(api.GetErrorString))dlsym(h, "ncclGetErrorString");
    api.ok = api.GetUniqueId && api.CommInitRank && api.AllReduce &&
             api.AllGather && api.CommDestroy && api.GetErrorString;
  });
  return &api;
}

extern "C" int l3g_nccl_unique_id(uint8_t out[128]) {
  NcclApi* api = nccl();
  if (!api->ok) return l3g_fail(L3G_E_NCCL, "libnccl.so.2 not found");
  ncclUniqueId id;
  NCCL_TRY(api->GetUniqueId(&id));
  static_assert(sizeof(id) == 128, "ncclUniqueId size");
  memcpy(out, &id, 128);
  return L3G_OK;
}


// ---------------------------------------------------------------------------
// kernel set-up
// ---------------------------------------------------------------------------
int sm_count(int dev) {
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 1;
}


// ---------------------------------------------------------------------------
// failure-detection self test
// ---------------------------------------------------------------------------
extern "C" int l3g_selftest_bounded_wait(int32_t device, int32_t timeout_us, int32_t* status) {
  if (!status) return l3g_fail(L3G_E_INVALID, "null argument");
  if (timeout_us <= 0 || timeout_us > 1000000)
    return l3g_fail(L3G_E_INVALID, "timeout_us must be in (0, 1e6]");
  int dev = device;
  if (dev < 0) CUDA_TRY(cudaGetDevice(&dev));
  CUDA_TRY(cudaSetDevice(dev));
  Result* d = nullptr;
  CUDA_TRY(cudaMalloc(&d, sizeof(Result)));
  cudaMemset(d, 0, sizeof(Result));
  k_selftest_wait<<<1, 32>>>(d, (unsigned long long)timeout_us * 1000ull);
  cudaError_t e = cudaDeviceSynchronize();
  Result h{};
  if (e == cudaSuccess) e = cudaMemcpy(&h, d, sizeof h, cudaMemcpyDeviceToHost);
  cudaFree(d);
  if (e != cudaSuccess) return l3g_fail(L3G_E_CUDA, "selftest: %s", cudaGetErrorString(e));
  *status = h.err == ERR_TIMEOUT ? L3G_E_DEVICE : (h.err ? -100 - h.err : L3G_OK);
  return L3G_OK;
}

