// extern "C" entry points of libfna2_b200.so (declared in include/fna2.h):
// argument validation, TMA tensor-map construction and kernel launches.
//
// The whole library is one translation unit (the kernel sources are included
// below) so the device-side watchdog flag needs no relocatable device code.
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <initializer_list>
#include <string>

#include "../../include/fna2.h"
#include "fna2_kernels.cuh"
#include "ptx.cuh"

#include "fna2_bwd.cu"
#include "fna2_fwd.cu"
#include "fna2_gemm.cu"
#include "fna2_qkprep.cu"
#include "fna2_decode.cu"

namespace fna2 {
namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define FNA2_CHECK(cond, ...) \
  do {                        \
    if (!(cond)) return fail(FNA2_ERR_INVALID, __VA_ARGS__); \
  } while (0)

#define FNA2_CUDA(call)                                                                     \
  do {                                                                                      \
    cudaError_t e_ = (call);                                                                \
    if (e_ != cudaSuccess) return fail(FNA2_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

// Driver-API calls (tensor-map encoding) need the device's primary context to
// be current on the calling thread; PyTorch's autograd worker threads may not
// have bound it yet.  cudaFree(nullptr) makes the runtime bind it.
int ensure_context() {
  thread_local bool bound = false;
  if (!bound) {
    cudaError_t e = cudaFree(nullptr);
    if (e != cudaSuccess) return fail(FNA2_ERR_CUDA, "cudaFree(nullptr): %s", cudaGetErrorString(e));
    bound = true;
  }
  return FNA2_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 4-D bf16 tensor map over (col, row, head, batch) with a (box0 x box1 x 1 x 1) box.
int make_map(CUtensorMap* m, const void* ptr, uint64_t cols, uint64_t rows, uint64_t heads, uint64_t batch,
             int64_t s_row, int64_t s_head, int64_t s_batch, uint32_t box0, uint32_t box1,
             CUtensorMapSwizzle swz, const char* what) {
  if (int rc = ensure_context()) return rc;
  auto enc = encode_fn();
  FNA2_CHECK(enc != nullptr, "cuTensorMapEncodeTiled is unavailable from the driver");
  // size-1 dimensions may carry any stride in PyTorch; give TMA a legal one
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

int check_tensor(const Fna2Tensor& t, const char* name, bool varlen) {
  FNA2_CHECK(t.ptr != nullptr, "%s: null pointer", name);
  FNA2_CHECK((reinterpret_cast<uintptr_t>(t.ptr) & 15u) == 0, "%s: base pointer must be 16-byte aligned", name);
  FNA2_CHECK(t.stride[3] == 1, "%s: column stride must be 1 (got %lld)", name, (long long)t.stride[3]);
  for (int i = varlen ? 1 : 0; i < 3; ++i)
    FNA2_CHECK(t.stride[i] >= 0 && (t.stride[i] % 8) == 0,
               "%s: stride[%d] = %lld must be a non-negative multiple of 8 elements (16 bytes)", name, i,
               (long long)t.stride[i]);
  return FNA2_OK;
}

struct Shape {
  bool varlen;
  int B, Sq, Sk, Tq, Tk, H, HKV, HG, D, r, RP;
  int rows_q() const { return varlen ? Tq : Sq; }
  int rows_k() const { return varlen ? Tk : Sk; }
  int batch_dim() const { return varlen ? 1 : B; }
};

int check_problem(const Fna2Problem& p, Shape* s) {
  s->varlen = p.cu_seqlens_q != nullptr;
  FNA2_CHECK((p.cu_seqlens_q == nullptr) == (p.cu_seqlens_k == nullptr),
             "cu_seqlens_q and cu_seqlens_k must both be given or both be NULL");
  FNA2_CHECK(p.batch >= 0 && p.seqlen_q >= 0 && p.seqlen_k >= 0, "negative batch or sequence length");
  FNA2_CHECK(p.head_dim == 64 || p.head_dim == 128, "head_dim must be 64 or 128 (got %d)", p.head_dim);
  FNA2_CHECK(p.heads > 0 && p.heads_kv > 0 && p.heads % p.heads_kv == 0,
             "heads (%d) must be a positive multiple of heads_kv (%d)", p.heads, p.heads_kv);
  FNA2_CHECK(p.heads_graph >= 0 && p.heads_graph <= p.heads, "heads_graph (%d) must be in [0, heads=%d]",
             p.heads_graph, p.heads);
  FNA2_CHECK(p.heads <= 65535 && p.batch <= 65535, "heads and batch/sequence count must be <= 65535");
  if (p.heads_graph > 0)
    FNA2_CHECK(p.rank > 0 && p.rank <= 32 && p.rank % 8 == 0, "rank must be 8, 16, 24 or 32 (got %d)", p.rank);
  FNA2_CHECK(p.softmax_scale > 0.f, "softmax_scale must be positive");
  if (s->varlen) FNA2_CHECK(p.total_q >= 0 && p.total_k >= 0, "negative total_q/total_k");
  s->B = p.batch;
  s->Sq = p.seqlen_q;
  s->Sk = p.seqlen_k;
  s->Tq = p.total_q;
  s->Tk = p.total_k;
  s->H = p.heads;
  s->HKV = p.heads_kv;
  s->HG = p.heads_graph;
  s->D = p.head_dim;
  s->r = p.heads_graph > 0 ? p.rank : 16;
  s->RP = s->r <= 16 ? 16 : 32;
  if (!s->varlen) FNA2_CHECK(p.seqlen_q == p.seqlen_k, "dense problems need seqlen_q == seqlen_k");
  return FNA2_OK;
}

// Grid order of the varlen kernels.  They launch one CTA per (table entry,
// head); each sequence's entries are listed heaviest causal tile first.  With
// the entry as the fast grid dimension (the default) the CTAs resident together
// work on one head of one sequence and share its streamed K/V (or Q/dO) tiles
// in L2, which matters when there are thousands of CTAs per SM.  On a small
// problem the same order dispatches the last heads' heaviest tiles in the last
// wave, and the kernel waits for them; with the head as the fast dimension
// every head's heaviest tiles go first.  Small: at most kHeadFastTokenHeads
// token-heads (rows x heads) and a table that fits the grid's y dimension.
constexpr int64_t kHeadFastTokenHeads = 768 * 1024;
bool head_fast_grid(const Shape& s) {
  if (!s.varlen) return false;
  const int64_t rows = s.Tq > s.Tk ? s.Tq : s.Tk;
  const int64_t tab = (rows + 127) / 128 + s.B;  // longest table: one entry per 128-row tile, plus one per sequence
  return rows * s.H <= kHeadFastTokenHeads && tab <= 65535;
}

ProblemDev to_dev(const Fna2Problem& p, const Shape& s) {
  ProblemDev d;
  d.heads = s.H;
  d.heads_kv = s.HKV;
  d.heads_graph = s.HG;
  d.head_dim = s.D;
  d.rank = s.r;
  d.seqlen_q = s.Sq;
  d.seqlen_k = s.Sk;
  d.total_q = s.varlen ? s.Tq : s.Sq;
  d.total_k = s.varlen ? s.Tk : s.Sk;
  d.varlen = s.varlen ? 1 : 0;
  d.causal = s.varlen ? 1 : (p.causal ? 1 : 0);
  d.head_fast = head_fast_grid(s) ? 1 : 0;
  d.cu_q = p.cu_seqlens_q;
  d.cu_k = p.cu_seqlens_k;
  d.scale = p.softmax_scale;
  d.scale_log2 = p.softmax_scale * kLog2e;
  d.gs = nullptr;
  return d;
}

// Tensor maps shared by forward and backward: Q/K/V (and dO) with 64-column
// SW128 boxes of 128 rows, R_q/R_k with r_pad-column boxes (zero-filled past r).
int map_qkv(CUtensorMap* m, const Fna2Tensor& t, const Shape& s, int rows, int heads, const char* what) {
  return make_map(m, t.ptr, s.D, rows, heads, s.batch_dim(), t.stride[2], t.stride[1], t.stride[0], 64, 128,
                  CU_TENSOR_MAP_SWIZZLE_128B, what);
}
// The backward kernels stream their non-stationary operand in tiles of
// box_rows rows (query tiles of dkdv_query_rows rows in the key-stationary
// kernel, dq_key_rows-row key tiles in the query-stationary one) and read the streamed
// R as a 64-column SW128 atom beside it (columns past r zero-filled).
int map_qkv_tile(CUtensorMap* m, const Fna2Tensor& t, const Shape& s, int rows, int heads, int box_rows,
                 const char* what) {
  return make_map(m, t.ptr, s.D, rows, heads, s.batch_dim(), t.stride[2], t.stride[1], t.stride[0], 64, box_rows,
                  CU_TENSOR_MAP_SWIZZLE_128B, what);
}
int map_r_tile(CUtensorMap* m, const Fna2Tensor& t, const Shape& s, int rows, int box_rows, const char* what) {
  return make_map(m, t.ptr, s.r, rows, s.HG, s.batch_dim(), t.stride[2], t.stride[1], t.stride[0], 64, box_rows,
                  CU_TENSOR_MAP_SWIZZLE_128B, what);
}
int map_r(CUtensorMap* m, const Fna2Tensor& t, const Shape& s, int rows, const char* what) {
  return make_map(m, t.ptr, s.r, rows, s.HG, s.batch_dim(), t.stride[2], t.stride[1], t.stride[0], s.RP, 128,
                  s.RP == 16 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B, what);
}

}  // namespace
}  // namespace fna2

using namespace fna2;

extern "C" int fna2_abi_version(void) { return FNA2_ABI_VERSION; }

extern "C" int fna2_gemm(const Fna2GemmArgs* a, void* stream) {
  g_last_error.clear();
  FNA2_CHECK(a != nullptr, "null args");
  FNA2_CHECK(a->m >= 1 && a->n >= 1 && a->k >= 1, "m, n, k must be >= 1 (got %lld, %lld, %lld)", (long long)a->m,
             (long long)a->n, (long long)a->k);
  FNA2_CHECK(a->m < (1ll << 31) && a->n < (1ll << 31) && a->k < (1ll << 31), "m, n, k must be < 2^31");
  FNA2_CHECK(a->n % 32 == 0, "n must be a multiple of 32 (got %lld)", (long long)a->n);
  FNA2_CHECK(a->c_dtype == FNA2_DTYPE_BF16 || a->c_dtype == FNA2_DTYPE_F32, "c_dtype must be bf16 or f32");
  FNA2_CHECK(a->split_k >= 1 && a->split_k <= 4096, "split_k must be in [1, 4096]");
  FNA2_CHECK(a->split_k == 1 || a->c_dtype == FNA2_DTYPE_F32, "split_k > 1 needs fp32 output");
  FNA2_CHECK(a->a != nullptr && a->b != nullptr && a->c != nullptr, "null operand pointer");
  FNA2_CHECK(((reinterpret_cast<uintptr_t>(a->a) | reinterpret_cast<uintptr_t>(a->b) | reinterpret_cast<uintptr_t>(a->c)) &
              15u) == 0,
             "operands must be 16-byte aligned");
  FNA2_CHECK(a->lda % 8 == 0 && a->ldb % 8 == 0, "lda and ldb must be multiples of 8 elements");
  FNA2_CHECK(a->ldc % (a->c_dtype == FNA2_DTYPE_F32 ? 4 : 8) == 0, "ldc must keep rows 16-byte aligned");
  FNA2_CHECK(a->lda >= (a->a_mn_major ? a->m : a->k) && a->ldb >= (a->b_mn_major ? a->n : a->k) && a->ldc >= a->n,
             "a leading dimension is smaller than its row");
  CUtensorMap ta, tb;
  // K-major: (k, rows) with 64 x tile-row boxes; MN-major: (rows, k) with 64 x 64 boxes
  if (a->a_mn_major) {
    if (int rc = make_map(&ta, a->a, a->m, a->k, 1, 1, a->lda, 0, 0, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B, "a")) return rc;
  } else {
    if (int rc = make_map(&ta, a->a, a->k, a->m, 1, 1, a->lda, 0, 0, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B, "a"))
      return rc;
  }
  // each CTA of a pair loads 128 rows of A and 128 rows (output columns) of B per tile
  if (a->b_mn_major) {
    if (int rc = make_map(&tb, a->b, a->n, a->k, 1, 1, a->ldb, 0, 0, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B, "b")) return rc;
  } else {
    if (int rc = make_map(&tb, a->b, a->k, a->n, 1, 1, a->ldb, 0, 0, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B, "b"))
      return rc;
  }
  GemmParams p;
  p.M = a->m;
  p.N = a->n;
  p.K = a->k;
  p.a_mn = a->a_mn_major ? 1 : 0;
  p.b_mn = a->b_mn_major ? 1 : 0;
  p.c = a->c;
  p.ldc = a->ldc;
  p.c_f32 = a->c_dtype == FNA2_DTYPE_F32 ? 1 : 0;
  p.chunks = static_cast<int>((a->k + kGemmBK - 1) / kGemmBK);
  const int split = a->split_k < p.chunks ? a->split_k : p.chunks;
  p.chunks_per_split = (p.chunks + split - 1) / split;
  p.tiles_n = static_cast<int>((a->n + kGemmBN - 1) / kGemmBN);
  const int64_t tiles = p.tiles_n * ((a->m + kGemmBM - 1) / kGemmBM);
  FNA2_CHECK(tiles * split < (1ll << 31), "too many output tiles");
  p.tiles = static_cast<int>(tiles);
  p.items = p.tiles * split;
  FNA2_CUDA(launch_gemm(ta, tb, p, static_cast<cudaStream_t>(stream)));
  return FNA2_OK;
}

extern "C" const char* fna2_last_error(void) { return g_last_error.c_str(); }

extern "C" int fna2_device_status(int reset) {
  int v = 0;
  FNA2_CUDA(cudaDeviceSynchronize());
  FNA2_CUDA(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)));
  if (reset) {
    int z = 0;
    FNA2_CUDA(cudaMemcpyToSymbol(g_device_error, &z, sizeof(int)));
  }
  return v;
}

extern "C" int fna2_debug_watchdog(int withhold_site, unsigned long long wait_limit_ns) {
  g_last_error.clear();
  FNA2_CHECK(withhold_site == 0 || withhold_site == kSiteFwdPFull, "withhold_site must be 0 or %d", kSiteFwdPFull);
  const uint64_t limit = wait_limit_ns ? static_cast<uint64_t>(wait_limit_ns) : kWaitTimeoutNs;
  FNA2_CUDA(cudaDeviceSynchronize());
  FNA2_CUDA(cudaMemcpyToSymbol(g_wait_limit_ns, &limit, sizeof(limit)));
  FNA2_CUDA(cudaMemcpyToSymbol(g_debug_withhold, &withhold_site, sizeof(int)));
  return FNA2_OK;
}

extern "C" int fna2_fwd(const Fna2FwdArgs* a, void* stream) {
  g_last_error.clear();
  FNA2_CHECK(a != nullptr, "null args");
  Shape s;
  if (int rc = check_problem(a->prob, &s)) return rc;
  if (s.B == 0 || s.Sq == 0 || s.H == 0) return FNA2_OK;
  if (int rc = check_tensor(a->q, "q", s.varlen)) return rc;
  if (int rc = check_tensor(a->k, "k", s.varlen)) return rc;
  if (int rc = check_tensor(a->v, "v", s.varlen)) return rc;
  if (int rc = check_tensor(a->out, "out", s.varlen)) return rc;
  FNA2_CHECK(a->lse != nullptr, "lse: null pointer");
  if (s.HG > 0) {
    if (int rc = check_tensor(a->r_q, "r_q", s.varlen)) return rc;
    if (int rc = check_tensor(a->r_k, "r_k", s.varlen)) return rc;
    FNA2_CHECK(a->graph_scale != nullptr, "graph_scale: null pointer");
  }
  if (s.varlen) {  // the table of real query-tile pairs
    const size_t need = fwd_workspace_bytes(true, s.rows_q(), s.B);
    if (a->workspace_bytes < need || a->workspace == nullptr)
      return fail(FNA2_ERR_WORKSPACE, "forward workspace too small: %zu < %zu bytes", a->workspace_bytes, need);
    FNA2_CHECK((reinterpret_cast<uintptr_t>(a->workspace) & 255u) == 0, "workspace must be 256-byte aligned");
  }
  CUtensorMap tq, tk, tv, trq, trk;
  if (int rc = map_qkv(&tq, a->q, s, s.rows_q(), s.H, "q")) return rc;
  if (int rc = map_qkv(&tk, a->k, s, s.rows_k(), s.HKV, "k")) return rc;
  if (int rc = map_qkv(&tv, a->v, s, s.rows_k(), s.HKV, "v")) return rc;
  if (s.HG > 0) {
    if (int rc = map_r(&trq, a->r_q, s, s.rows_q(), "r_q")) return rc;
    if (int rc = map_r(&trk, a->r_k, s, s.rows_k(), "r_k")) return rc;
  } else {
    trq = tq;  // never dereferenced: no graph heads
    trk = tk;
  }
  FwdParams p;
  p.prob = to_dev(a->prob, s);
  p.prob.gs = a->graph_scale;
  p.out = static_cast<__nv_bfloat16*>(a->out.ptr);
  p.o_sb = s.varlen ? 0 : a->out.stride[0];
  p.o_sh = a->out.stride[1];
  p.o_sr = a->out.stride[2];
  p.lse = a->lse;
  p.lse_sbh = s.rows_q();
  p.n_mblocks = (s.Sq + kBlockM - 1) / kBlockM;
  p.tab = s.varlen ? static_cast<int4*>(a->workspace) : nullptr;
  p.tab_len = s.varlen ? fwd_tab_len(s.rows_q(), s.B) : 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaEvent_t* ev = reinterpret_cast<cudaEvent_t*>(a->launch_events);
  if (ev) FNA2_CUDA(cudaEventRecord(ev[0], st));
  FNA2_CUDA(launch_fwd(s.D, s.RP, tq, tk, tv, trq, trk, p, s.H, s.B, st));
  if (ev) FNA2_CUDA(cudaEventRecord(ev[1], st));
  return FNA2_OK;
}

extern "C" size_t fna2_fwd_workspace_size(const Fna2Problem* prob) {
  if (!prob) return 0;
  Shape s;
  if (check_problem(*prob, &s)) return 0;
  return fwd_workspace_bytes(s.varlen, s.rows_q(), s.B);
}

extern "C" size_t fna2_bwd_workspace_size(const Fna2Problem* prob) {
  if (!prob) return 0;
  Shape s;
  if (check_problem(*prob, &s)) return 0;
  return bwd_workspace_bytes(s.batch_dim(), s.H, s.HG, s.rows_q(), s.varlen, s.rows_k(), s.B);
}

namespace fna2 {
namespace {

// Argument checks shared by fna2_bwd and fna2_bwd_noalloc.  *empty is set when
// the problem has no rows (nothing to launch).
int bwd_check_args(const Fna2BwdArgs* a, Shape* s, bool* empty) {
  FNA2_CHECK(a != nullptr, "null args");
  if (int rc = check_problem(a->prob, s)) return rc;
  *empty = s->B == 0 || s->Sq == 0;
  if (*empty) return FNA2_OK;
  const char* names[] = {"q", "k", "v", "out", "dout", "dq", "dk", "dv"};
  const Fna2Tensor* ts[] = {&a->q, &a->k, &a->v, &a->out, &a->dout, &a->dq, &a->dk, &a->dv};
  for (int i = 0; i < 8; ++i)
    if (int rc = check_tensor(*ts[i], names[i], s->varlen)) return rc;
  FNA2_CHECK(a->lse != nullptr, "lse: null pointer");
  if (s->HG > 0) {
    if (int rc = check_tensor(a->r_q, "r_q", s->varlen)) return rc;
    if (int rc = check_tensor(a->r_k, "r_k", s->varlen)) return rc;
    if (int rc = check_tensor(a->dr_q, "dr_q", s->varlen)) return rc;
    if (int rc = check_tensor(a->dr_k, "dr_k", s->varlen)) return rc;
    FNA2_CHECK(a->graph_scale != nullptr && a->d_graph_scale != nullptr, "graph_scale/d_graph_scale: null");
  }
  return FNA2_OK;
}

size_t bwd_scratch_bytes(const Shape& s) {
  return bwd_workspace_bytes(s.batch_dim(), s.H, s.HG, s.rows_q(), s.varlen, s.rows_k(), s.B);
}

// Tensor maps and kernel parameters of a checked backward call, with `scratch`
// (bwd_scratch_bytes(s) bytes, 256-byte aligned) as its workspace; then the
// three launches on `stream`.
int bwd_launch(const Fna2BwdArgs* a, const Shape& s, void* scratch, void* stream) {
  BwdMaps m;
  if (int rc = map_qkv(&m.q, a->q, s, s.rows_q(), s.H, "q")) return rc;
  if (int rc = map_qkv(&m.k, a->k, s, s.rows_k(), s.HKV, "k")) return rc;
  if (int rc = map_qkv(&m.v, a->v, s, s.rows_k(), s.HKV, "v")) return rc;
  if (int rc = map_qkv(&m.dO, a->dout, s, s.rows_q(), s.H, "dout")) return rc;
  const int qs_rows = dkdv_query_rows(s.D, s.RP);
  if (int rc = map_qkv_tile(&m.qS, a->q, s, s.rows_q(), s.H, qs_rows, "q")) return rc;
  if (int rc = map_qkv_tile(&m.dOS, a->dout, s, s.rows_q(), s.H, qs_rows, "dout")) return rc;
  const int kd_rows = dq_key_rows(s.D, s.RP);
  if (int rc = map_qkv_tile(&m.kDq, a->k, s, s.rows_k(), s.HKV, kd_rows, "k")) return rc;
  if (int rc = map_qkv_tile(&m.vDq, a->v, s, s.rows_k(), s.HKV, kd_rows, "v")) return rc;
  if (s.HG > 0) {
    if (int rc = map_r(&m.rq, a->r_q, s, s.rows_q(), "r_q")) return rc;
    if (int rc = map_r(&m.rk, a->r_k, s, s.rows_k(), "r_k")) return rc;
    if (int rc = map_r_tile(&m.rqS, a->r_q, s, s.rows_q(), qs_rows, "r_q")) return rc;
    if (int rc = map_r_tile(&m.rkDq, a->r_k, s, s.rows_k(), kd_rows, "r_k")) return rc;
  } else {
    m.rq = m.q;  // never dereferenced: no graph heads
    m.rk = m.k;
    m.rqS = m.qS;
    m.rkDq = m.kDq;
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
  FNA2_CUDA(launch_bwd(s.D, s.RP, m, p, static_cast<cudaStream_t>(stream),
                       reinterpret_cast<cudaEvent_t*>(a->launch_events)));
  return FNA2_OK;
}

}  // namespace
}  // namespace fna2

extern "C" int fna2_bwd(const Fna2BwdArgs* a, void* stream) {
  g_last_error.clear();
  Shape s;
  bool empty = false;
  if (int rc = bwd_check_args(a, &s, &empty)) return rc;
  if (empty) return FNA2_OK;
  const size_t need = bwd_scratch_bytes(s);
  if (a->workspace_bytes < need || (need && a->workspace == nullptr))
    return fail(FNA2_ERR_WORKSPACE, "workspace too small: %zu < %zu bytes", a->workspace_bytes, need);
  FNA2_CHECK((reinterpret_cast<uintptr_t>(a->workspace) & 255u) == 0, "workspace must be 256-byte aligned");
  return bwd_launch(a, s, a->workspace, stream);
}

// The no-allocation backward entry point (fna2_bwd_noalloc) and its static scratch.
#include "fna2_noalloc.cu"

// ---------------------------------------------------------------------------
// varlen QK-RMSNorm + RoPE
// ---------------------------------------------------------------------------
namespace fna2 {
namespace {

int check_rows(const Fna2Rows& r, int heads, int elem_bytes, int D, const char* what) {
  if (heads == 0) return FNA2_OK;
  FNA2_CHECK(r.ptr != nullptr, "%s: null pointer", what);
  FNA2_CHECK(reinterpret_cast<uintptr_t>(r.ptr) % 16 == 0, "%s: base pointer must be 16-byte aligned", what);
  const int64_t vec = 16 / elem_bytes;
  FNA2_CHECK(r.token_stride % vec == 0 && r.head_stride % vec == 0,
             "%s: token/head strides must be multiples of %lld elements", what, static_cast<long long>(vec));
  FNA2_CHECK(r.token_stride >= 0 && r.head_stride >= 0, "%s: negative stride", what);
  (void)D;
  return FNA2_OK;
}

int qk_prep_params(const Fna2QkPrepArgs* a, QkPrepParams* p) {
  FNA2_CHECK(a != nullptr, "null arguments");
  FNA2_CHECK(a->head_dim == 64 || a->head_dim == 128, "head_dim must be 64 or 128 (got %d)", a->head_dim);
  FNA2_CHECK(a->total_tokens >= 0 && a->heads_q >= 0 && a->heads_k >= 0, "negative size");
  FNA2_CHECK(a->in_dtype == FNA2_DTYPE_F32 || a->in_dtype == FNA2_DTYPE_BF16, "bad in_dtype %d", a->in_dtype);
  FNA2_CHECK(a->weight_dtype == FNA2_DTYPE_F32 || a->weight_dtype == FNA2_DTYPE_BF16, "bad weight_dtype %d",
             a->weight_dtype);
  FNA2_CHECK(a->rope_dtype == FNA2_DTYPE_F32 || a->rope_dtype == FNA2_DTYPE_BF16, "bad rope_dtype %d", a->rope_dtype);
  FNA2_CHECK((a->q_weight == nullptr) == (a->k_weight == nullptr), "set both RMSNorm weights or neither");
  FNA2_CHECK(a->eps >= 0.f, "eps must be >= 0");
  if (a->inv_freq) FNA2_CHECK(a->cu_seqlens != nullptr && a->num_seqs >= 1, "RoPE needs cu_seqlens with >= 1 sequence");
  const int in_bytes = a->in_dtype == FNA2_DTYPE_BF16 ? 2 : 4;
  if (int rc = check_rows(a->q_in, a->heads_q, in_bytes, a->head_dim, "q_in")) return rc;
  if (int rc = check_rows(a->k_in, a->heads_k, in_bytes, a->head_dim, "k_in")) return rc;
  std::memset(p, 0, sizeof(*p));
  p->T = a->total_tokens;
  p->N = a->num_seqs;
  p->cu = a->cu_seqlens;
  p->hq = a->heads_q;
  p->hk = a->heads_k;
  p->in_bf16 = a->in_dtype == FNA2_DTYPE_BF16;
  p->w_bf16 = a->weight_dtype == FNA2_DTYPE_BF16;
  p->rope_bf16 = a->rope_dtype == FNA2_DTYPE_BF16;
  p->qi = {const_cast<void*>(a->q_in.ptr), a->q_in.token_stride, a->q_in.head_stride};
  p->ki = {const_cast<void*>(a->k_in.ptr), a->k_in.token_stride, a->k_in.head_stride};
  p->qw = a->q_weight;
  p->kw = a->k_weight;
  p->eps = a->eps;
  p->inv_freq = a->inv_freq;
  return FNA2_OK;
}

}  // namespace
}  // namespace fna2

extern "C" int fna2_qk_prep_fwd(const Fna2QkPrepArgs* a, void* stream) {
  QkPrepParams p;
  if (int rc = qk_prep_params(a, &p)) return rc;
  if (int rc = check_rows(a->q_out, a->heads_q, 2, a->head_dim, "q_out")) return rc;
  if (int rc = check_rows(a->k_out, a->heads_k, 2, a->head_dim, "k_out")) return rc;
  p.qo = {a->q_out.ptr, a->q_out.token_stride, a->q_out.head_stride};
  p.ko = {a->k_out.ptr, a->k_out.token_stride, a->k_out.head_stride};
  if (p.T == 0 || p.hq + p.hk == 0) return FNA2_OK;
  FNA2_CUDA(launch_qk_prep(p, a->head_dim, false, static_cast<cudaStream_t>(stream)));
  return FNA2_OK;
}

extern "C" int fna2_qk_prep_bwd(const Fna2QkPrepBwdArgs* b, void* stream) {
  FNA2_CHECK(b != nullptr, "null arguments");
  const Fna2QkPrepArgs* a = &b->fwd;
  QkPrepParams p;
  if (int rc = qk_prep_params(a, &p)) return rc;
  const int in_bytes = a->in_dtype == FNA2_DTYPE_BF16 ? 2 : 4;
  if (int rc = check_rows(b->dq_out, a->heads_q, 2, a->head_dim, "dq_out")) return rc;
  if (int rc = check_rows(b->dk_out, a->heads_k, 2, a->head_dim, "dk_out")) return rc;
  if (int rc = check_rows(b->dq_in, a->heads_q, in_bytes, a->head_dim, "dq_in")) return rc;
  if (int rc = check_rows(b->dk_in, a->heads_k, in_bytes, a->head_dim, "dk_in")) return rc;
  if (a->q_weight) FNA2_CHECK(b->dq_weight != nullptr && b->dk_weight != nullptr, "weight gradients needed");
  p.dqo = {const_cast<void*>(b->dq_out.ptr), b->dq_out.token_stride, b->dq_out.head_stride};
  p.dko = {const_cast<void*>(b->dk_out.ptr), b->dk_out.token_stride, b->dk_out.head_stride};
  p.dqi = {b->dq_in.ptr, b->dq_in.token_stride, b->dq_in.head_stride};
  p.dki = {b->dk_in.ptr, b->dk_in.token_stride, b->dk_in.head_stride};
  p.dqw = a->q_weight ? b->dq_weight : nullptr;
  p.dkw = a->q_weight ? b->dk_weight : nullptr;
  if (p.T == 0 || p.hq + p.hk == 0) return FNA2_OK;
  FNA2_CUDA(launch_qk_prep(p, a->head_dim, true, static_cast<cudaStream_t>(stream)));
  return FNA2_OK;
}

namespace {

int decode_num_splits(const Fna2DecodeArgs* a, int head_blocks) {
  if (a->num_splits > 0) return a->num_splits;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t ctas = static_cast<int64_t>(a->batch) * a->kv_heads * head_blocks;
  const int64_t want = (4LL * sms + ctas - 1) / std::max<int64_t>(ctas, 1);  // about two waves of two CTAs per SM
  const int64_t cap = std::max<int64_t>(1, (a->capacity + 255) / 256);     // at least 256 keys per split
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({want, cap, 64})));
}

int decode_params(const Fna2DecodeArgs* a, DecodeParams* p, int* D_out, size_t* smem) {
  FNA2_CHECK(a != nullptr, "null arguments");
  FNA2_CHECK(a->head_dim == 64 || a->head_dim == 128, "head_dim must be 64 or 128 (got %d)", a->head_dim);
  FNA2_CHECK(a->batch >= 0 && a->heads >= 0 && a->kv_heads > 0 && a->capacity >= 0, "bad sizes");
  FNA2_CHECK(a->heads % a->kv_heads == 0, "heads (%d) must be a multiple of kv_heads (%d)", a->heads, a->kv_heads);
  FNA2_CHECK(a->graph_heads >= 0 && a->graph_heads <= a->heads, "graph_heads must be in [0, heads]");
  if (a->graph_heads > 0) {
    FNA2_CHECK(a->rank == 16 || a->rank == 32, "rank must be 16 or 32 (got %d)", a->rank);
    FNA2_CHECK(a->r_q && a->rk_cache && a->graph_scale, "graph heads need r_q, rk_cache and graph_scale");
  }
  FNA2_CHECK(a->softmax_scale > 0.f, "softmax_scale must be positive");
  FNA2_CHECK(a->q && a->k_cache && a->v_cache && a->out && a->cache_seqlens, "null tensor pointer");
  const bool has_new = a->k_new != nullptr;
  FNA2_CHECK(has_new == (a->v_new != nullptr), "k_new and v_new go together");
  if (has_new && a->graph_heads > 0) FNA2_CHECK(a->rk_new != nullptr, "k_new with graph heads needs rk_new");
  auto al = [](const void* ptr) { return reinterpret_cast<uintptr_t>(ptr) % 16 == 0; };
  auto st8 = [](std::initializer_list<int64_t> v) {
    for (int64_t x : v)
      if (x < 0 || x % 8) return false;
    return true;
  };
  FNA2_CHECK(al(a->q) && al(a->k_cache) && al(a->v_cache) && al(a->out) && (!a->r_q || al(a->r_q)) &&
                 (!a->rk_cache || al(a->rk_cache)) && (!has_new || (al(a->k_new) && al(a->v_new))) &&
                 (!a->rk_new || al(a->rk_new)),
             "tensor base pointers must be 16-byte aligned");
  FNA2_CHECK(st8({a->q_batch_stride, a->q_head_stride, a->k_batch_stride, a->k_token_stride, a->k_head_stride,
                  a->v_batch_stride, a->v_token_stride, a->v_head_stride, a->out_batch_stride, a->out_head_stride,
                  a->rq_batch_stride, a->rq_head_stride, a->rk_batch_stride, a->rk_token_stride, a->rk_head_stride,
                  a->kn_batch_stride, a->kn_head_stride, a->vn_batch_stride, a->vn_head_stride,
                  a->rkn_batch_stride, a->rkn_head_stride}),
             "strides must be non-negative multiples of 8 elements");
  DecodeParams& d = *p;
  d = DecodeParams{};
  d.B = a->batch, d.H = a->heads, d.HKV = a->kv_heads, d.HG = a->graph_heads, d.R = a->graph_heads ? a->rank : 16;
  d.G = a->heads / a->kv_heads, d.capacity = a->capacity;
  d.scale = a->softmax_scale, d.scale_log2 = a->softmax_scale * 1.4426950408889634f;
  using bf = __nv_bfloat16;
  d.q = static_cast<const bf*>(a->q), d.q_sb = a->q_batch_stride, d.q_sh = a->q_head_stride;
  d.rq = static_cast<const bf*>(a->r_q), d.rq_sb = a->rq_batch_stride, d.rq_sh = a->rq_head_stride;
  d.kc = static_cast<bf*>(a->k_cache), d.k_sb = a->k_batch_stride, d.k_st = a->k_token_stride, d.k_sh = a->k_head_stride;
  d.vc = static_cast<bf*>(a->v_cache), d.v_sb = a->v_batch_stride, d.v_st = a->v_token_stride, d.v_sh = a->v_head_stride;
  d.rkc = static_cast<bf*>(a->rk_cache), d.rk_sb = a->rk_batch_stride, d.rk_st = a->rk_token_stride;
  d.rk_sh = a->rk_head_stride;
  d.gs = a->graph_scale, d.seqlens = a->cache_seqlens, d.offsets = a->cache_offsets;
  d.kn = static_cast<const bf*>(a->k_new), d.kn_sb = a->kn_batch_stride, d.kn_sh = a->kn_head_stride;
  d.vn = static_cast<const bf*>(a->v_new), d.vn_sb = a->vn_batch_stride, d.vn_sh = a->vn_head_stride;
  d.rkn = static_cast<const bf*>(a->rk_new), d.rkn_sb = a->rkn_batch_stride, d.rkn_sh = a->rkn_head_stride;
  d.out = static_cast<bf*>(a->out), d.o_sb = a->out_batch_stride, d.o_sh = a->out_head_stride;
  d.lse = a->lse;
  d.head_blocks = (d.G + 15) / 16;
  d.splits = decode_num_splits(a, d.head_blocks);
  const int ng_max = std::min(16, std::min(d.G, d.HG));
  d.stages = decode_stages(a->head_dim, ng_max, d.R);
  *smem = decode_smem_bytes(a->head_dim, ng_max, d.R, d.stages);
  *D_out = a->head_dim;
  return FNA2_OK;
}

}  // namespace

extern "C" size_t fna2_decode_workspace_size(const Fna2DecodeArgs* a) {
  g_last_error.clear();
  DecodeParams p;
  int D = 0;
  size_t smem = 0;
  if (decode_params(a, &p, &D, &smem) != FNA2_OK) return 0;
  return p.splits > 1 ? static_cast<size_t>(p.B) * p.H * p.splits * (D + 2) * sizeof(float) : 0;
}

extern "C" int fna2_decode(const Fna2DecodeArgs* a, void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  DecodeParams p;
  int D = 0;
  size_t smem = 0;
  if (int rc = decode_params(a, &p, &D, &smem)) return rc;
  if (p.B == 0 || p.H == 0) return FNA2_OK;
  const size_t need = p.splits > 1 ? static_cast<size_t>(p.B) * p.H * p.splits * (D + 2) * sizeof(float) : 0;
  if (need > 0) {
    if (workspace == nullptr || workspace_bytes < need)
      return fail(FNA2_ERR_WORKSPACE, "decode workspace: need %zu bytes, got %zu", need, workspace_bytes);
    FNA2_CHECK(reinterpret_cast<uintptr_t>(workspace) % 16 == 0, "workspace must be 16-byte aligned");
    p.ws = static_cast<float*>(workspace);
  }
  FNA2_CUDA(launch_decode(p, D, smem, static_cast<cudaStream_t>(stream)));
  return FNA2_OK;
}
