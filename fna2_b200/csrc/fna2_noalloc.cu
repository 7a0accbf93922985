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
// routine; the kernels and their launch configuration are those of fna2_bwd.
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

// Tensor map without the context binding of make_map (the symbol lookup above
// has already made the device's context current on this thread).
int noalloc_map(CUtensorMap* m, const void* ptr, uint64_t cols, uint64_t rows, uint64_t heads, uint64_t batch,
                int64_t s_row, int64_t s_head, int64_t s_batch, uint32_t box0, uint32_t box1, CUtensorMapSwizzle swz,
                const char* what) {
  auto enc = encode_fn();
  FNA2_CHECK(enc != nullptr, "cuTensorMapEncodeTiled is unavailable from the driver");
  if (rows <= 1 && (s_row <= 0 || (s_row * 2) % 16)) s_row = 8;
  if (heads <= 1 && (s_head <= 0 || (s_head * 2) % 16)) s_head = s_row * static_cast<int64_t>(rows ? rows : 1);
  if (batch <= 1 && (s_batch <= 0 || (s_batch * 2) % 16)) s_batch = s_head * static_cast<int64_t>(heads ? heads : 1);
  cuuint64_t dims[4] = {cols, rows ? rows : 1, heads ? heads : 1, batch ? batch : 1};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(s_row) * 2, static_cast<cuuint64_t>(s_head) * 2,
                           static_cast<cuuint64_t>(s_batch) * 2};
  cuuint32_t box[4] = {box0, box1, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FNA2_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (%d) for %s", static_cast<int>(r), what);
  return FNA2_OK;
}

}  // namespace
}  // namespace fna2

extern "C" int fna2_bwd_noalloc(const Fna2BwdArgs* a, void* stream) {
  using namespace fna2;
  g_last_error.clear();
  FNA2_CHECK(a != nullptr, "null args");
  Shape s;
  if (int rc = check_problem(a->prob, &s)) return rc;
  if (s.B == 0 || s.Sq == 0) return FNA2_OK;
  const char* names[] = {"q", "k", "v", "out", "dout", "dq", "dk", "dv"};
  const Fna2Tensor* ts[] = {&a->q, &a->k, &a->v, &a->out, &a->dout, &a->dq, &a->dk, &a->dv};
  for (int i = 0; i < 8; ++i)
    if (int rc = check_tensor(*ts[i], names[i], s.varlen)) return rc;
  FNA2_CHECK(a->lse != nullptr, "lse: null pointer");
  if (s.HG > 0) {
    if (int rc = check_tensor(a->r_q, "r_q", s.varlen)) return rc;
    if (int rc = check_tensor(a->r_k, "r_k", s.varlen)) return rc;
    if (int rc = check_tensor(a->dr_q, "dr_q", s.varlen)) return rc;
    if (int rc = check_tensor(a->dr_k, "dr_k", s.varlen)) return rc;
    FNA2_CHECK(a->graph_scale != nullptr && a->d_graph_scale != nullptr, "graph_scale/d_graph_scale: null");
  }
  const size_t need = bwd_workspace_bytes(s.batch_dim(), s.H, s.HG, s.rows_q(), s.varlen, s.rows_k(), s.B);
  if (need > static_cast<size_t>(FNA2_NOALLOC_SCRATCH_BYTES))
    return fail(FNA2_ERR_WORKSPACE,
                "fna2_bwd_noalloc: problem needs %zu bytes of scratch (8 bytes per query row and head, "
                "batch*heads*rows = %lld, plus the tile tables of packed batches) but the static scratch holds "
                "%d bytes; use fna2_bwd with a workspace",
                need, static_cast<long long>(s.batch_dim()) * s.H * s.rows_q(), FNA2_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;

  auto map_t = [&](CUtensorMap* m, const Fna2Tensor& t, int rows, int heads, const char* what) {
    return noalloc_map(m, t.ptr, s.D, rows, heads, s.batch_dim(), t.stride[2], t.stride[1], t.stride[0], 64, 128,
                       CU_TENSOR_MAP_SWIZZLE_128B, what);
  };
  auto map_rr = [&](CUtensorMap* m, const Fna2Tensor& t, int rows, const char* what) {
    return noalloc_map(m, t.ptr, s.r, rows, s.HG, s.batch_dim(), t.stride[2], t.stride[1], t.stride[0], s.RP, 128,
                       s.RP == 16 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B, what);
  };
  auto map_tt = [&](CUtensorMap* m, const Fna2Tensor& t, int rows, int heads, int box_rows, const char* what) {
    return noalloc_map(m, t.ptr, s.D, rows, heads, s.batch_dim(), t.stride[2], t.stride[1], t.stride[0], 64,
                       box_rows, CU_TENSOR_MAP_SWIZZLE_128B, what);
  };
  auto map_rt = [&](CUtensorMap* m, const Fna2Tensor& t, int rows, int box_rows, const char* what) {
    return noalloc_map(m, t.ptr, s.r, rows, s.HG, s.batch_dim(), t.stride[2], t.stride[1], t.stride[0], 64,
                       box_rows, CU_TENSOR_MAP_SWIZZLE_128B, what);
  };
  const int qs_rows = dkdv_query_rows(s.D, s.RP);
  BwdMaps mp;
  if (int rc = map_t(&mp.q, a->q, s.rows_q(), s.H, "q")) return rc;
  if (int rc = map_t(&mp.k, a->k, s.rows_k(), s.HKV, "k")) return rc;
  if (int rc = map_t(&mp.v, a->v, s.rows_k(), s.HKV, "v")) return rc;
  if (int rc = map_t(&mp.dO, a->dout, s.rows_q(), s.H, "dout")) return rc;
  if (int rc = map_tt(&mp.qS, a->q, s.rows_q(), s.H, qs_rows, "q")) return rc;
  if (int rc = map_tt(&mp.dOS, a->dout, s.rows_q(), s.H, qs_rows, "dout")) return rc;
  if (int rc = map_tt(&mp.k112, a->k, s.rows_k(), s.HKV, kQT, "k")) return rc;
  if (int rc = map_tt(&mp.v112, a->v, s.rows_k(), s.HKV, kQT, "v")) return rc;
  if (s.HG > 0) {
    if (int rc = map_rr(&mp.rq, a->r_q, s.rows_q(), "r_q")) return rc;
    if (int rc = map_rr(&mp.rk, a->r_k, s.rows_k(), "r_k")) return rc;
    if (int rc = map_rt(&mp.rqS, a->r_q, s.rows_q(), qs_rows, "r_q")) return rc;
    if (int rc = map_rt(&mp.rk112, a->r_k, s.rows_k(), kQT, "r_k")) return rc;
  } else {
    mp.rq = mp.q;
    mp.rk = mp.k;
    mp.rqS = mp.qS;
    mp.rk112 = mp.k112;
  }
  BwdParams p;
  std::memset(&p, 0, sizeof(p));
  p.prob = to_dev(a->prob, s);
  p.prob.gs = a->graph_scale;
  auto set3 = [&](const Fna2Tensor& t, int64_t* sb, int64_t* sh, int64_t* sr) {
    *sb = s.varlen ? 0 : t.stride[0];
    *sh = t.stride[1];
    *sr = t.stride[2];
  };
  p.out = static_cast<const __nv_bfloat16*>(a->out.ptr);
  set3(a->out, &p.o_sb, &p.o_sh, &p.o_sr);
  p.dout = static_cast<const __nv_bfloat16*>(a->dout.ptr);
  set3(a->dout, &p.do_sb, &p.do_sh, &p.do_sr);
  p.q = static_cast<const __nv_bfloat16*>(a->q.ptr);
  set3(a->q, &p.q_sb, &p.q_sh, &p.q_sr);
  p.lse = a->lse;
  p.lse_sbh = s.rows_q();
  p.dq = static_cast<__nv_bfloat16*>(a->dq.ptr);
  set3(a->dq, &p.dq_sb, &p.dq_sh, &p.dq_sr);
  p.dk = static_cast<__nv_bfloat16*>(a->dk.ptr);
  set3(a->dk, &p.dk_sb, &p.dk_sh, &p.dk_sr);
  p.dv = static_cast<__nv_bfloat16*>(a->dv.ptr);
  set3(a->dv, &p.dv_sb, &p.dv_sh, &p.dv_sr);
  if (s.HG > 0) {
    p.drq = static_cast<__nv_bfloat16*>(a->dr_q.ptr);
    set3(a->dr_q, &p.drq_sb, &p.drq_sh, &p.drq_sr);
    p.drk = static_cast<__nv_bfloat16*>(a->dr_k.ptr);
    set3(a->dr_k, &p.drk_sb, &p.drk_sh, &p.drk_sr);
    p.rq = static_cast<const __nv_bfloat16*>(a->r_q.ptr);
    set3(a->r_q, &p.rq_sb, &p.rq_sh, &p.rq_sr);
    p.dgs = a->d_graph_scale;
  }
  p.total_q_rows = s.rows_q();
  p.total_k_rows = s.rows_k();
  p.batch = s.B;
  p.n_mblocks = (s.Sq + kBlockM - 1) / kBlockM;
  p.n_nblocks = (s.Sk + kBlockN - 1) / kBlockN;
  bwd_set_workspace(&p, scratch, s.batch_dim(), s.H, s.rows_q(), s.varlen, s.rows_k(), s.B);
  FNA2_CUDA(launch_bwd(s.D, s.RP, mp, p, static_cast<cudaStream_t>(stream),
                       reinterpret_cast<cudaEvent_t*>(a->launch_events)));
  return FNA2_OK;
}
