// Library-wide entry points: version, errors, device status, SM count, and the
// host helper that encodes TMA tensor maps through the driver entry point.
#include <cstdarg>
#include <cstring>
#include <mutex>

#include "mt_common.cuh"
#include "mt_tma.h"

namespace mt {

__device__ int g_device_status = 0;

static thread_local char g_err[1024] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

void clear_error() { g_err[0] = 0; }

int cuda_fail(cudaError_t e, const char* what) {
  set_error("%s failed: %s (%d)", what, cudaGetErrorString(e), static_cast<int>(e));
  return MT_ERR_CUDA;
}

namespace {
struct SmemAttr {
  const void* kernel;
  int dev;
  int bytes;
};
std::mutex g_smem_mu;
SmemAttr g_smem_attrs[512];
int g_smem_n = 0;
}  // namespace

int smem_attr_lookup(const void* kernel, int dev) {
  std::lock_guard<std::mutex> lock(g_smem_mu);
  for (int i = 0; i < g_smem_n; ++i)
    if (g_smem_attrs[i].kernel == kernel && g_smem_attrs[i].dev == dev) return g_smem_attrs[i].bytes;
  return 0;
}

void smem_attr_store(const void* kernel, int dev, int bytes) {
  std::lock_guard<std::mutex> lock(g_smem_mu);
  for (int i = 0; i < g_smem_n; ++i)
    if (g_smem_attrs[i].kernel == kernel && g_smem_attrs[i].dev == dev) {
      g_smem_attrs[i].bytes = bytes;
      return;
    }
  if (g_smem_n < 512) g_smem_attrs[g_smem_n++] = {kernel, dev, bytes};
}

int device_sm_count(int* out) {
  static int cached[64] = {0};
  int dev = 0;
  MT_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && cached[dev] > 0) {
    *out = cached[dev];
    return MT_OK;
  }
  int n = 0;
  MT_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  if (dev >= 0 && dev < 64) cached[dev] = n;
  *out = n;
  return MT_OK;
}

// ------------------------------------------------------------- tensor maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, int rank,
              const uint64_t* dims, const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return MT_ERR_CUDA;
  }
  if (rank < 2 || rank > 5) {
    set_error("tensor map: rank %d outside 2..5", rank);
    return MT_ERR_INVALID_ARGUMENT;
  }
  bool ok = aligned(base, 16) && (box[0] * elem_bytes) % 16 == 0;
  for (int i = 0; i + 1 < rank; ++i) ok = ok && strides[i] % 16 == 0;
  if (!ok) {
    set_error("tensor map: base %p / strides / box inner %u x %d B break the 16-byte rule", base, box[0],
              elem_bytes);
    return MT_ERR_INVALID_ARGUMENT;
  }
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], estr[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    estr[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) st[i] = strides[i];
  CUresult r = fn(map, dt, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, st, bx, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): rank %d, dims %llu x %llu, box %u x %u", (int)r, rank,
              (unsigned long long)dims[0], (unsigned long long)dims[1], box[0], box[1]);
    return MT_ERR_CUDA;
  }
  return MT_OK;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes,
                 uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  const uint64_t dims[2] = {inner, outer};
  const uint64_t strides[1] = {row_stride_bytes};
  const uint32_t box[2] = {box_inner, box_outer};
  return make_tmap(map, base, dt, elem_bytes, 2, dims, strides, box, swizzle);
}

}  // namespace mt

extern "C" {

int mt_version(void) { return (0 << 16) | (1 << 8) | 0; }

uint64_t mt_kernel_launches(void) { return mt::g_kernel_launches.load(std::memory_order_relaxed); }

const char* mt_last_error_string(void) { return mt::g_err; }

int mt_device_status(int* status_out, int clear) {
  if (!status_out) {
    mt::set_error("mt_device_status: status_out is NULL");
    return MT_ERR_INVALID_ARGUMENT;
  }
  MT_CUDA(cudaDeviceSynchronize());
  int v = 0;
  MT_CUDA(cudaMemcpyFromSymbol(&v, mt::g_device_status, sizeof(int)));
  if (clear) {
    int z = 0;
    MT_CUDA(cudaMemcpyToSymbol(mt::g_device_status, &z, sizeof(int)));
  }
  *status_out = v;
  return MT_OK;
}

int mt_sm_count(int* sm_count_out) {
  if (!sm_count_out) {
    mt::set_error("mt_sm_count: output is NULL");
    return MT_ERR_INVALID_ARGUMENT;
  }
  return mt::device_sm_count(sm_count_out);
}

}  // extern "C"
