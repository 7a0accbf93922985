// fna2_bwd_noalloc: the backward pass for callers that cannot allocate device
// memory.
//
// fna2_bwd needs a caller-provided scratch buffer (the log2-domain LSE and
// Delta = rowsum(dO*O) rows, 8 bytes per query row and head, plus for packed
// batches 32 bytes per query tile and per key tile).  Some callers
// cannot provide one: processes whose device memory is entirely owned by
// another allocator (a framework's caching pool or a fixed arena sized at
// start-up, where an extra cudaMalloc would fail or fragment the arena), and
// thin language bindings (cgo, JNI, ctypes) that only hand over tensors they
// already hold and have no allocator of their own to reach.  For them this
// entry point takes its scratch from a file-scope device array instead.
//
// Properties of that array (every GPU that loads the library holds it until
// the process exits):
//   - size FNA2_NOALLOC_SCRATCH_BYTES (32 MiB); problems needing more are
//     rejected with FNA2_ERR_WORKSPACE before any work is enqueued;
//   - one array per device, shared by every call on that device and keeping
//     the last call's contents.  Nothing in it has to start at zero: the
//     pre-pass overwrites every row the backward kernels read.  Calls whose
//     GPU work overlaps (different streams or host threads without ordering)
//     race on it and produce wrong gradients; order them on one stream;
//   - its device address is looked up with cudaGetSymbolAddress on the first
//     call made on each device (with that device current).  Make that first
//     call before any stream capture.
// The entry point itself calls no cudaMalloc, cudaFree or other allocating
// routine; its checks, tensor maps, kernels and launch configuration are
// fna2_bwd's own (bwd_check_args / bwd_launch in fna2_api.cu).
#include <mutex>

namespace fna2 {
namespace {

// File-scope scratch: host code must not pass `g_noalloc_scratch` itself to a
// kernel (in host code the name is a host-side stand-in, not a device
// address); the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[FNA2_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set-up once per device).
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(FNA2_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(FNA2_ERR_INVALID, "device ordinal %d >= %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess)
      return fail(FNA2_ERR_CUDA, "cudaGetSymbolAddress(scratch) on device %d: %s", dev, cudaGetErrorString(e));
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return FNA2_OK;
}

}  // namespace
}  // namespace fna2

extern "C" int fna2_bwd_noalloc(const Fna2BwdArgs* a, void* stream) {
  using namespace fna2;
  g_last_error.clear();
  Shape s;
  bool empty = false;
  if (int rc = bwd_check_args(a, &s, &empty)) return rc;
  if (empty) return FNA2_OK;
  const size_t need = bwd_scratch_bytes(s);
  if (need > static_cast<size_t>(FNA2_NOALLOC_SCRATCH_BYTES))
    return fail(FNA2_ERR_WORKSPACE,
                "fna2_bwd_noalloc: problem needs %zu bytes of scratch (8 bytes per query row and head, "
                "batch*heads*rows = %lld, plus the tile tables of packed batches) but the static scratch holds "
                "%d bytes; use fna2_bwd with a workspace",
                need, static_cast<long long>(s.batch_dim()) * s.H * s.rows_q(), FNA2_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  // same validation, tensor maps (make_map binds the device context on this
  // thread), parameters and launches as fna2_bwd; only the scratch differs
  return bwd_launch(a, s, scratch, stream);
}
