// INT4 paged decode attention for callers that cannot allocate device memory.
//
// iris_b200_int4_paged_decode needs scratch memory: per call it writes the
// sequences' page prefix sums and the split-KV partial records into a
// workspace the caller provides.  Some callers have no way to get one: code
// running inside a host framework that owns every device allocation and
// offers no allocation hook (an inference-server plugin or a foreign-language
// binding restricted to the tensors it is handed), code called from an
// allocator or a stream callback where cudaMalloc must not be called, or a
// serving loop that forbids allocation after start-up.  This file gives them
// iris_b200_int4_paged_decode_noalloc, which uses a fixed scratch array of
// IRIS_DECODE_NOALLOC_SCRATCH_BYTES that lives in the library itself.
//
// The array is a file-scope __device__ variable: every GPU on which the
// library is loaded holds it until the process exits.  In host code its name
// is only a host-side stand-in for the symbol, so the device address is
// obtained with cudaGetSymbolAddress once per device (on the first call made
// with that device current) and passed to the kernels.  All calls share the
// array and it keeps whatever the last call left; nothing in it has to start
// at zero (each call rewrites what it reads).  Calls whose work overlaps on
// the GPU (several streams, several host threads) race on the array.
#include <mutex>

#include "common.cuh"

// From decode.cu (library-internal, not exported): the workspace a decode
// needs when its page ranges are capped by the problem (batch *
// max_pages_per_seq pages at most, at least 4 pages per range) rather than by
// the GPU's SM count, and the INT4 decode entry that applies that cap.
size_t problem_workspace_bytes(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                               int32_t max_pages_per_seq, int32_t device);
int iris_decode_problem_sized(const void* query, const void* k_data, const void* v_data, const void* k_scale,
                              const void* v_scale, const int32_t* block_table, int64_t block_table_stride,
                              const int32_t* seq_lens, void* output, float* out_lse, int32_t out_mode, int32_t batch,
                              int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int64_t num_pages,
                              int32_t page_size, int32_t max_pages_per_seq, float softmax_scale, void* workspace,
                              size_t workspace_bytes, int32_t* error_word, void* stream);

namespace {

static __device__ __align__(256) unsigned char g_decode_scratch[IRIS_DECODE_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 128;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once
// per device).  Returns nullptr and records the CUDA error on failure.
void* scratch_on_device(int device) {
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[device] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
    if (e != cudaSuccess) {
      iris::record_cuda_error(e, "cudaGetSymbolAddress(decode scratch)");
      return nullptr;
    }
    g_scratch_ptr[device] = ptr;
  }
  return g_scratch_ptr[device];
}

}  // namespace

extern "C" int iris_b200_int4_paged_decode_noalloc(const void* query, const void* k_data, const void* v_data,
                                                   const void* k_scale, const void* v_scale,
                                                   const int32_t* block_table, int64_t block_table_stride,
                                                   const int32_t* seq_lens, void* output, float* out_lse,
                                                   int32_t out_mode, int32_t batch, int32_t num_q_heads,
                                                   int32_t num_kv_heads, int32_t head_dim, int64_t num_pages,
                                                   int32_t page_size, int32_t max_pages_per_seq,
                                                   float softmax_scale, int32_t* error_word, void* stream) {
  int device = 0;
  const cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) {
    iris::record_cuda_error(e, "cudaGetDevice");
    return IRIS_ECUDA;
  }
  if (device < 0 || device >= kMaxDevices) return IRIS_EUNSUPPORTED;
  // The problem must fit the static array; the size is checked before the
  // array is touched.  The split-KV ranges are capped by the problem's page
  // count (not only by the SM count), so small problems need little scratch.
  const size_t need =
      problem_workspace_bytes(batch, num_q_heads, num_kv_heads, head_dim, max_pages_per_seq, device);
  if (batch > 0 && need == 0) return IRIS_EINVAL;
  if (need > static_cast<size_t>(IRIS_DECODE_NOALLOC_SCRATCH_BYTES)) return IRIS_EWORKSPACE;
  void* scratch = scratch_on_device(device);
  if (scratch == nullptr) return IRIS_ECUDA;
  return iris_decode_problem_sized(query, k_data, v_data, k_scale, v_scale, block_table, block_table_stride,
                                   seq_lens, output, out_lse, out_mode, batch, num_q_heads, num_kv_heads, head_dim,
                                   num_pages, page_size, max_pages_per_seq, softmax_scale, scratch,
                                   static_cast<size_t>(IRIS_DECODE_NOALLOC_SCRATCH_BYTES), error_word, stream);
}
