// Host-side plumbing of the C ABI: last-error messages, reading the device
// error word, SM counts and a small cache of TMA tensor maps.
#pragma once
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "nb_common.cuh"

namespace {

thread_local char g_msg[512] = "";

constexpr int kMaxDevices = 64;
std::mutex g_mu;
int g_sms[kMaxDevices] = {};

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

struct MapKey {
  const void* base;
  int dtype;
  uint64_t cols, rows, stride;
  uint32_t box_cols, box_rows;
  int device;
  bool operator==(const MapKey& o) const {
    return base == o.base && dtype == o.dtype && cols == o.cols && rows == o.rows &&
           stride == o.stride && box_cols == o.box_cols && box_rows == o.box_rows &&
           device == o.device;
  }
};
constexpr int kMapCache = 256;
struct MapEntry {
  MapKey key;
  CUtensorMap map;
  bool used;
};
MapEntry g_maps[kMapCache];
int g_map_next = 0;

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

}  // namespace

namespace nbh {

// Launch configuration with programmatic stream serialisation (programmatic
// dependent launch): the grid may be scheduled while the previous kernel in
// the stream drains; its kernels call griddep_wait() before reading anything.
inline bool pdl_enabled() {
  static int on = [] {
    const char* e = getenv("NB_PDL");  // "0" launches without the attribute (diagnostics)
    return (e && e[0] == '0') ? 0 : 1;
  }();
  return on != 0;
}

inline void pdl_config(cudaLaunchConfig_t& cfg, cudaLaunchAttribute (&attr)[1], dim3 grid,
                       dim3 block, size_t smem, cudaStream_t st) {
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
}


int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(NB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return NB_OK;
}

int num_sms() {
  const int d = current_device();
  if (d < 0 || d >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_sms[d]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
    g_sms[d] = n > 0 ? n : 148;
  }
  return g_sms[d];
}

int ensure_max_smem(const void* func, int bytes, const char* what) {
  struct Entry {
    const void* func;
    int device;
    int bytes;
  };
  static Entry table[512];
  static int used = 0;
  const int d = current_device();
  std::lock_guard<std::mutex> lk(g_mu);
  for (int i = 0; i < used; ++i)
    if (table[i].func == func && table[i].device == d && table[i].bytes >= bytes) return NB_OK;
  const cudaError_t e =
      cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess)
    return fail(NB_ERR_CUDA, "%s: shared-memory attribute: %s", what, cudaGetErrorString(e));
  for (int i = 0; i < used; ++i)
    if (table[i].func == func && table[i].device == d) {
      table[i].bytes = bytes;
      return NB_OK;
    }
  if (used < 512) table[used++] = Entry{func, d, bytes};
  return NB_OK;
}

int tensor_map_2d(CUtensorMap* out, const void* base, int dtype, uint64_t cols, uint64_t rows,
                  uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows) {
  const MapKey key{base, dtype, cols, rows, row_stride_bytes, box_cols, box_rows,
                   current_device()};
  std::lock_guard<std::mutex> lk(g_mu);
  for (int i = 0; i < kMapCache; ++i) {
    if (g_maps[i].used && g_maps[i].key == key) {
      *out = g_maps[i].map;
      return NB_OK;
    }
  }
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e =
        cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
      return fail(NB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  CUtensorMapDataType dt = dtype == NB_DTYPE_BF16   ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                           : dtype == NB_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMap map;
  CUresult r = g_encode(&map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(NB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for %llux%llu stride %llu", (int)r,
                (unsigned long long)rows, (unsigned long long)cols,
                (unsigned long long)row_stride_bytes);
  g_maps[g_map_next] = MapEntry{key, map, true};
  g_map_next = (g_map_next + 1) % kMapCache;
  *out = map;
  return NB_OK;
}

}  // namespace nbh

extern "C" {

int nb_abi_version(void) { return 3; }

const char* nb_last_error(void) { return g_msg; }

int nb_device_errors(unsigned* flags_out) {
  if (!flags_out) return nbh::fail(NB_ERR_INVALID_ARG, "flags_out is NULL");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return nbh::fail(NB_ERR_CUDA, "device error: %s", cudaGetErrorString(e));
  unsigned v = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&v, nb::g_error_word, sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(nb::g_error_word, &zero, sizeof(unsigned));
  if (e != cudaSuccess)
    return nbh::fail(NB_ERR_CUDA, "reading the error word: %s", cudaGetErrorString(e));
  *flags_out = v;
  return NB_OK;
}

}  // extern "C"
