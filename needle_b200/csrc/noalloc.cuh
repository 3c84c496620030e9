// nb_paged_decode_noalloc: paged decode for callers that cannot allocate
// device memory.
//
// nb_paged_decode needs a caller-provided workspace for its split-K partial
// results.  Some callers have no way to provide one: a host bound through a
// plain FFI (Go, Java, Rust, ...) that has no device allocator of its own and
// no torch tensor to lend; a serving loop that must not call cudaMalloc
// between launches because cudaMalloc can synchronise the device; or a
// deployment whose device memory is budgeted once at start-up.  This variant
// takes the same arguments minus the workspace and keeps the partials in a
// fixed array in the library's own device memory instead.
//
// The array is a file-scope __device__ array of NB_NOALLOC_SCRATCH_BYTES, so
// every GPU that loads the library holds it until the process exits.  Host
// code cannot use the array's name as a device address (it is a host-side
// stand-in); the entry point looks the real address up with
// cudaGetSymbolAddress once per device, on the first call made on that
// device with that device current.  Make that first call before any stream
// capture.  Every call shares the one array and it keeps the last call's
// contents; the split kernel writes every partial the merge kernel reads in
// the same call, so nothing needs clearing.  Calls that overlap on the GPU
// (different streams, or different host threads on one device) race on the
// array and must be serialised by the caller.  No cudaMalloc, cudaFree or
// allocating library routine is called.
#pragma once
#include <mutex>

#include "nb_common.cuh"

namespace nb {
__device__ __align__(256) unsigned char g_noalloc_scratch[NB_NOALLOC_SCRATCH_BYTES];
}  // namespace nb

namespace nbh {

// Device address of nb::g_noalloc_scratch on the current device, looked up
// once per device.  Returns nullptr (with the message set) on failure.
inline void* noalloc_scratch() {
  static std::mutex mu;
  static void* addr[64] = {};
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    fail(NB_ERR_CUDA, "nb_paged_decode_noalloc: no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, nb::g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      fail(NB_ERR_CUDA, "nb_paged_decode_noalloc: cudaGetSymbolAddress failed: %s",
           cudaGetErrorString(e));
      return nullptr;
    }
    addr[dev] = p;
  }
  return addr[dev];
}

}  // namespace nbh

extern "C" {

int nb_paged_decode_noalloc(const void* q, int64_t q_stride_seq, int64_t q_stride_head,
                            const void* kv_cache, int num_blocks, int num_kv_heads,
                            int block_size, int head_dim, int num_q_heads,
                            const int32_t* block_table, int64_t block_table_stride,
                            int max_blocks_per_seq, const int32_t* context_lens, int num_seqs,
                            float scale, void* out, int64_t out_stride_seq,
                            int64_t out_stride_head, int pages_per_split, int dtype,
                            void* stream) {
  using namespace nbh;
  if (pages_per_split <= 0) return fail(NB_ERR_INVALID_ARG, "pages_per_split must be > 0");
  if (num_seqs <= 0 || num_q_heads <= 0 || head_dim <= 0 || max_blocks_per_seq <= 0)
    return nb_paged_decode(q, q_stride_seq, q_stride_head, kv_cache, num_blocks, num_kv_heads,
                           block_size, head_dim, num_q_heads, block_table, block_table_stride,
                           max_blocks_per_seq, context_lens, num_seqs, scale, out,
                           out_stride_seq, out_stride_head, nullptr, 0, pages_per_split, dtype,
                           stream);
  const int max_splits = (max_blocks_per_seq + pages_per_split - 1) / pages_per_split;
  const size_t need = nb_paged_decode_workspace_size(num_seqs, num_q_heads, head_dim, max_splits);
  if (need > (size_t)NB_NOALLOC_SCRATCH_BYTES)
    return fail(NB_ERR_INVALID_ARG,
                "nb_paged_decode_noalloc: this shape needs %zu bytes of split-K scratch but the "
                "fixed scratch holds %zu; use larger pages_per_split, a smaller batch, or "
                "nb_paged_decode with a caller-allocated workspace",
                need, (size_t)NB_NOALLOC_SCRATCH_BYTES);
  void* ws = nullptr;
  if (need > 0) {
    ws = noalloc_scratch();
    if (!ws) return NB_ERR_CUDA;
  }
  return nb_paged_decode(q, q_stride_seq, q_stride_head, kv_cache, num_blocks, num_kv_heads,
                         block_size, head_dim, num_q_heads, block_table, block_table_stride,
                         max_blocks_per_seq, context_lens, num_seqs, scale, out, out_stride_seq,
                         out_stride_head, ws, (size_t)NB_NOALLOC_SCRATCH_BYTES, pages_per_split,
                         dtype, stream);
}

}  // extern "C"
