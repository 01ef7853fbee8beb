// mj_decode_noalloc: the split-KV decode for callers that cannot allocate
// device memory.
//
// Who needs it: a serving engine that has already handed every spare byte of
// HBM to its own pre-sized KV-cache pool (so a later cudaMalloc would fail or
// fragment it), code that issues the decode while a stream is being captured
// into a CUDA graph in global capture mode (where cudaMalloc is an illegal
// call), and plugin hosts whose interface passes a plugin only its input and
// output buffers. Such a caller cannot provide the split-KV partial buffers
// (o_part / lse_part) that mj_decode takes from its caller.
//
// This entry point takes them from a fixed array compiled into the library
// instead: kNoallocScratchBytes (16 MiB) of device memory that every GPU which
// loads the library holds until the process exits. It allocates nothing
// itself -- no cudaMalloc, cudaFree or allocating library routine.
//
// Set-up: the first call on each device looks up the device address of the
// array (cudaGetSymbolAddress with that device current) and caches it; make
// that first call before any stream capture begins. Later calls only read
// the cached address. The address belongs to the device's primary context
// as it was at that first call: after cudaDeviceReset (or any reset of the
// primary context) the module loads again, possibly elsewhere, and the
// cached address is stale -- a process that resets a device must not call
// this entry point on it again.
//
// Sharing: every call on a device uses the same array, which keeps whatever
// the previous call left in it. Nothing needs to start at zero: the decode
// writes every partial row before the combine reads it. Two calls that run
// at the same time on the GPU (different streams, no ordering) race on the
// array and corrupt each other's partials; order them.
#include <stdio.h>

#include <mutex>

#include "common.cuh"

namespace mj {
int set_last_error(int code, const char* msg);
}  // namespace mj

namespace {

constexpr size_t kNoallocScratchBytes = size_t(16) << 20;  // 16 MiB per device
constexpr int kMaxDevices = 64;

// The partials live here: o_part first, lse_part after it (both fp32).
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {};

int setup_device(int dev, void** out) {
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    // host code must ask the runtime for the device address of the array
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return (int)e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return 0;
}

}  // namespace

extern "C" int mj_decode(const mj_decode_args* args, void* stream);

extern "C" int mj_decode_noalloc(const mj_decode_args* args, void* stream) {
  if (!args) return mj::set_last_error(MJ_ERR_INVALID, "mj_decode_noalloc: null args");
  mj_decode_args a = *args;
  const int n_q = a.q_len * (a.h_k > 0 ? a.h_q / a.h_k : 0);
  const size_t rows = (size_t)(a.max_splits > 0 ? a.max_splits : 0) * (size_t)(a.num_seqs > 0 ? a.num_seqs : 0) *
                      (size_t)(a.h_k > 0 ? a.h_k : 0) * (size_t)(n_q > 0 ? n_q : 0);
  const size_t o_bytes = rows * (size_t)(a.head_size > 0 ? a.head_size : 0) * sizeof(float);
  const size_t need = o_bytes + rows * sizeof(float);
  if (need > kNoallocScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "mj_decode_noalloc: split-KV partials need %zu bytes (max_splits %d x num_seqs %d x h_k %d x %d rows "
             "x (head_size + 1) x 4 B) but the built-in scratch holds %zu; lower max_splits or use mj_decode",
             need, a.max_splits, a.num_seqs, a.h_k, n_q, kNoallocScratchBytes);
    return mj::set_last_error(MJ_ERR_UNSUPPORTED, msg);
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return mj::set_last_error(MJ_ERR_CUDA, "mj_decode_noalloc: no usable current device");
  void* base = nullptr;
  int e = setup_device(dev, &base);
  if (e != 0) {
    char msg[160];
    snprintf(msg, sizeof(msg), "mj_decode_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString((cudaError_t)e));
    return mj::set_last_error(MJ_ERR_CUDA, msg);
  }
  a.o_part = reinterpret_cast<float*>(base);
  a.lse_part = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(base) + o_bytes);
  a.part_seqs = a.num_seqs;
  a.with_combine = 1;  // the partials are internal, so the merge always runs here
  return mj_decode(&a, stream);
}
