// Host utilities shared by every launcher: the driver's tensor-map encoder (looked up once through
// the runtime, so the library needs no link-time dependency on libcuda) and the SM count.
#include <mutex>

#include "gemm_tc.cuh"

namespace noise {

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int device_sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 1;
}

int make_tmap_2d(CUtensorMap* map, const void* ptr, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                 uint64_t cols, uint64_t row_stride_elems, uint32_t box_rows, uint32_t box_cols) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return 1;
  if (box_cols * elem_bytes != 128) return 1;  // one 128-byte swizzle row per box row
  if ((row_stride_elems * elem_bytes) % 16 != 0) return 1;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : 1;
}

}  // namespace noise

// ------------------------------------------------------------------------------------------------
// Launch accounting and optional per-kernel timing. Every kernel launch of the library goes through
// LaunchScope, which counts it and, while profiling is on, brackets it with CUDA events on the
// launching stream so the host can read per-kind device times afterwards.
// ------------------------------------------------------------------------------------------------
#include <atomic>
#include <vector>

#include "profile.cuh"

namespace noise {

static std::atomic<long long> g_launches{0};

struct ProfRecord {
  int kind;
  cudaEvent_t a, b;
};

static struct {
  std::mutex mu;
  bool on = false;
  std::vector<cudaEvent_t> pool;
  size_t used = 0;
  std::vector<ProfRecord> recs;
} g_prof;

static cudaEvent_t pool_event() {
  if (g_prof.used == g_prof.pool.size()) {
    cudaEvent_t e;
    cudaEventCreate(&e);
    g_prof.pool.push_back(e);
  }
  return g_prof.pool[g_prof.used++];
}

LaunchScope::LaunchScope(int kind, cudaStream_t s, int kernels) : kind_(kind), s_(s), idx_(-1) {
  g_launches.fetch_add(kernels, std::memory_order_relaxed);
  std::lock_guard<std::mutex> lk(g_prof.mu);
  if (!g_prof.on) return;
  ProfRecord r{kind, pool_event(), pool_event()};
  cudaEventRecord(r.a, s);
  idx_ = (int)g_prof.recs.size();
  g_prof.recs.push_back(r);
}

LaunchScope::~LaunchScope() {
  if (idx_ < 0) return;
  std::lock_guard<std::mutex> lk(g_prof.mu);
  cudaEventRecord(g_prof.recs[idx_].b, s_);
}

}  // namespace noise

using namespace noise;

extern "C" int64_t noise_launch_count(void) { return g_launches.load(); }

extern "C" int noise_profile_enable(int on) {
  std::lock_guard<std::mutex> lk(g_prof.mu);
  g_prof.on = on != 0;
  g_prof.recs.clear();
  g_prof.used = 0;
  return kStatusOk;
}

extern "C" int noise_profile_read(double* ms, int64_t* count, int kinds) {
  std::lock_guard<std::mutex> lk(g_prof.mu);
  for (int k = 0; k < kinds; ++k) ms[k] = 0.0, count[k] = 0;
  for (const ProfRecord& r : g_prof.recs) {
    if (r.kind < 0 || r.kind >= kinds) continue;
    if (cudaEventSynchronize(r.b) != cudaSuccess) return kStatusLaunchFailed;
    float t = 0.f;
    cudaEventElapsedTime(&t, r.a, r.b);
    ms[r.kind] += t;
    count[r.kind] += 1;
  }
  return kStatusOk;
}
