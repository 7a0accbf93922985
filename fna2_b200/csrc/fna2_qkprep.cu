// Varlen QK-RMSNorm + RoPE pre-attention transform (forward and backward).
//
// Reference semantics: FNA2/attention_fna2.py RMSNorm.forward (:100-102):
// n = x * rsqrt(mean(x^2) + eps) * w; RotaryPositionalEmbedding (:108-163):
// y = n*cos + rotate_half(n)*sin with cos/sin = cos/sin(cat(t*f, t*f)), the
// table built in the dtype of the rotated tensor (:148-155); and
// _apply_rope_varlen (:620-647): t restarts at 0 for every packed sequence.
//
// HBM-bound elementwise work.  Each warp owns a contiguous run of tokens and
// streams the rows (token, head) of that run through a small ring of
// asynchronous copies in shared memory; a row is spread over head_dim/16 lanes
// so that both halves of every rotate_half pair sit in one lane.  A token's
// position comes from a warp-wide search over cu_seqlens (skipped while the
// run stays inside one sequence) and its cos/sin values are computed once and
// reused for all of its heads.  The backward recomputes the norm and reduces
// the weight gradients per warp, then per CTA, then with one atomic per
// column and CTA.
#include "fna2_kernels.cuh"

namespace fna2 {

struct QkRows {
  void* ptr;
  int64_t ts, hs;  // token, head strides (elements)
};

struct QkPrepParams {
  int64_t T;
  int N;
  const int* cu;
  int hq, hk;
  int in_bf16, w_bf16, rope_bf16;
  QkRows qi, ki, qo, ko;            // inputs (in dtype), outputs (bf16)
  QkRows dqo, dko, dqi, dki;        // backward: grads of outputs (bf16), grads of inputs (in dtype)
  const void* qw;
  const void* kw;
  float eps;
  const float* inv_freq;
  float* dqw;
  float* dkw;
};

constexpr int kPrepThreads = 256;
constexpr int kRowBatch = 2;     // row instructions per streamed unit (forward)
constexpr int kRowBatchBwd = 1;  // the same for the backward (twice the operands per row)

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Layout: a row (one token, one head, D values) is spread over LPR = D/16 lanes;
// lane `sub` of a row holds the 8 values [8*sub, 8*sub+8) of the first half and
// the 8 values [D/2 + 8*sub, ...) of the second half, so the rotate_half pairs
// (e, e + D/2) sit in the same lane and RoPE needs no shuffles; row sums reduce
// over the row's LPR lanes.  A warp covers RPW = 32/LPR rows per instruction.
// Inputs stream through a per-warp ring of asynchronous copies (kPrepStages row
// batches deep); each lane reads back only the 16-byte pieces it copied.
constexpr int kHPL = 8;         // values per lane per half row
constexpr int kPrepStages = 4;  // row batches in flight per warp

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Copy this lane's two half-row pieces (8 values each) of one row into dst.
__device__ __forceinline__ void stage_row(uint8_t* dst, const void* base, int64_t row_off, int D, int sub,
                                          int in_bytes, bool valid) {
  const uint8_t* b = static_cast<const uint8_t*>(base);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint8_t* src = b + (row_off + h * (D / 2) + kHPL * sub) * in_bytes;
    uint8_t* d = dst + h * kHPL * in_bytes;
    cp_async16(d, valid ? src : b, valid);
    if (in_bytes == 4) cp_async16(d + 16, valid ? src + 16 : b, valid);
  }
}

// Read back the staged pieces as x1 (first half) and x2 (second half).
__device__ __forceinline__ void unstage_row(const uint8_t* src, bool is_bf16, float (&x1)[kHPL], float (&x2)[kHPL]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float* x = h ? x2 : x1;
    if (is_bf16) {
      const uint4 w = *reinterpret_cast<const uint4*>(src + h * kHPL * 2);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ww[i]));
        x[2 * i] = f.x, x[2 * i + 1] = f.y;
      }
    } else {
      const float4* f4 = reinterpret_cast<const float4*>(src + h * kHPL * 4);
      const float4 a = f4[0], b = f4[1];
      x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
    }
  }
}

__device__ __forceinline__ void store_half(void* base, int64_t off, bool is_bf16, const float (&y)[kHPL]) {
  if (is_bf16) {
    uint4 w;
    w.x = pack_bf16(y[0], y[1]);
    w.y = pack_bf16(y[2], y[3]);
    w.z = pack_bf16(y[4], y[5]);
    w.w = pack_bf16(y[6], y[7]);
    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(base) + off) = w;
  } else {
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(base) + off);
    p[0] = make_float4(y[0], y[1], y[2], y[3]);
    p[1] = make_float4(y[4], y[5], y[6], y[7]);
  }
}

// Sequence bounds [*lo, *hi) of token t (all lanes of the warp call it with the
// same t); returns false if t belongs to no sequence.  A 32-way search: each
// round the lanes probe 32 evenly spaced cu_seqlens entries.
__device__ __forceinline__ bool warp_find_sequence(const QkPrepParams& p, int64_t t, int lane, int* lo_out,
                                                   int* hi_out) {
  if (t < __ldg(p.cu) || t >= __ldg(p.cu + p.N)) return false;
  int lo = 0, hi = p.N;  // cu[lo] <= t < cu[hi]
  while (hi - lo > 1) {
    const int step = (hi - lo + 31) / 32;
    const int idx = min(lo + lane * step, hi);
    const bool le = idx < hi && __ldg(p.cu + idx) <= t;
    const unsigned m = __ballot_sync(0xffffffffu, le);
    const int last = 31 - __clz(m);  // lane 0 always qualifies
    lo = lo + last * step;
    hi = min(lo + step, hi);
  }
  *lo_out = __ldg(p.cu + lo);
  *hi_out = __ldg(p.cu + lo + 1);
  return true;
}

// cos/sin of this lane's 8 frequencies at position pos, formed as the reference
// forms its table: fp32 t*f, or (bf16 mode) t, f and t*f rounded to bf16 and
// cos/sin rounded to bf16.
__device__ __forceinline__ void rope_table(const QkPrepParams& p, int pos, int sub, float (&c)[kHPL],
                                           float (&s)[kHPL]) {
#pragma unroll
  for (int v = 0; v < kHPL; ++v) {
    const float f = __ldg(p.inv_freq + kHPL * sub + v), t = static_cast<float>(pos);
    const float ang = p.rope_bf16 ? bf16_round(bf16_round(t) * bf16_round(f)) : t * f;
    sincosf(ang, &s[v], &c[v]);
    if (p.rope_bf16) {
      c[v] = bf16_round(c[v]);
      s[v] = bf16_round(s[v]);
    }
  }
}

template <int LPR, int N>
__device__ __forceinline__ void row_sums(float (&v)[N]) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1)
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
}

// Shared-memory layout of both directions: the two RMSNorm weights (fp32) and,
// per warp, kPrepStages units of row batches (x, and dy for the backward).
inline size_t qk_prep_smem(int D, int in_bytes, bool bwd) {
  const int rows_per_unit = (bwd ? kRowBatchBwd : kRowBatch) * 32 / (D / (2 * kHPL));
  return static_cast<size_t>(2 * D * 4) + static_cast<size_t>(kPrepThreads / 32) * kPrepStages * rows_per_unit * D *
                                              in_bytes * (bwd ? 2 : 1);
}

// One kernel for both directions: BWD reads x and dy and writes dx (+ weight
// gradients); the forward reads x and writes y.
template <int D, bool BWD>
__global__ void __launch_bounds__(kPrepThreads) fna2_qk_prep_kernel(const QkPrepParams p) {
  constexpr int LPR = D / (2 * kHPL), RPW = 32 / LPR;
  constexpr int RBATCH = BWD ? kRowBatchBwd : kRowBatch;
  constexpr int RB = RPW * RBATCH;                 // rows per streamed unit
  constexpr int OPS = BWD ? 2 : 1;
  extern __shared__ __align__(16) uint8_t prep_smem[];
  float* s_w = reinterpret_cast<float*>(prep_smem);  // [2][D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sub = lane % LPR, rsel = lane / LPR;
  const bool rope = p.inv_freq != nullptr, norm = p.qw != nullptr;
  const int rows = p.hq + p.hk, units_per_token = (rows + RB - 1) / RB;
  const int in_bytes = p.in_bf16 ? 2 : 4;
  const int row_bytes = D * in_bytes;                 // one row of one operand, all lanes of the row
  const int unit_bytes = RB * row_bytes * OPS;
  uint8_t* wbuf = prep_smem + 2 * D * 4 + static_cast<size_t>(warp) * kPrepStages * unit_bytes;
  if (norm)
    for (int e = threadIdx.x; e < 2 * D; e += kPrepThreads) {
      const void* w = e < D ? p.qw : p.kw;
      const int i = e % D;
      s_w[e] = p.w_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(w)[i]) : static_cast<const float*>(w)[i];
    }
  __syncthreads();
  float gq1[kHPL], gq2[kHPL], gk1[kHPL], gk2[kHPL];  // weight gradients (backward)
#pragma unroll
  for (int v = 0; v < kHPL; ++v) gq1[v] = gq2[v] = gk1[v] = gk2[v] = 0.f;

  const int64_t nw = static_cast<int64_t>(gridDim.x) * (kPrepThreads / 32);
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * (kPrepThreads / 32) + warp;
  const int64_t chunk = (p.T + nw - 1) / nw;
  const int64_t run_beg = gw * chunk, run_end = min(p.T, run_beg + chunk);
  const int64_t n_units = run_end > run_beg ? (run_end - run_beg) * units_per_token : 0;
  // lane slot of row batch j within a unit: [operand][j][lane] pieces of 2*kHPL values
  auto slot = [&](uint8_t* st, int op, int j) { return st + ((op * RBATCH + j) * 32 + lane) * 2 * kHPL * in_bytes; };
  auto issue = [&](int64_t u) {
    if (u < n_units) {
      const int64_t t = run_beg + u / units_per_token;
      const int b = static_cast<int>(u % units_per_token);
      uint8_t* st = wbuf + (u % kPrepStages) * unit_bytes;
#pragma unroll
      for (int j = 0; j < RBATCH; ++j) {
        const int r = b * RB + j * RPW + rsel;
        const bool valid = r < rows, isq = r < p.hq;
        const int hh = isq ? r : r - p.hq;
        if (BWD) {
          const QkRows& go = isq ? p.dqo : p.dko;
          stage_row(slot(st, 0, j), go.ptr, t * go.ts + hh * go.hs, D, sub, 2, valid);
          if (norm) {
            const QkRows& in = isq ? p.qi : p.ki;
            stage_row(slot(st, 1, j), in.ptr, t * in.ts + hh * in.hs, D, sub, in_bytes, valid);
          }
        } else {
          const QkRows& in = isq ? p.qi : p.ki;
          stage_row(slot(st, 0, j), in.ptr, t * in.ts + hh * in.hs, D, sub, in_bytes, valid);
        }
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int u = 0; u < kPrepStages - 1; ++u) issue(u);
  int s_lo = 0, s_hi = 0;
  bool inside = true;
  float c[kHPL], s[kHPL];
  for (int64_t u = 0; u < n_units; ++u) {
    issue(u + kPrepStages - 1);
    cp_async_wait<kPrepStages - 1>();  // unit u has landed
    const int64_t t = run_beg + u / units_per_token;
    const int b = static_cast<int>(u % units_per_token);
    if (b == 0 && rope) {  // a new token: its position and cos/sin
      if (t < s_lo || t >= s_hi) {
        inside = warp_find_sequence(p, t, lane, &s_lo, &s_hi);
        if (!inside) s_lo = s_hi = 0;
      }
      if (inside) rope_table(p, static_cast<int>(t - s_lo), sub, c, s);
    }
    uint8_t* st = wbuf + (u % kPrepStages) * unit_bytes;
    if (!BWD) {
      if (rope && !inside) continue;  // outside every sequence: left unset, as the reference does
      float x1[RBATCH][kHPL], x2[RBATCH][kHPL], ss[RBATCH];
#pragma unroll
      for (int j = 0; j < RBATCH; ++j) unstage_row(slot(st, 0, j), p.in_bf16, x1[j], x2[j]);
      if (norm) {
#pragma unroll
        for (int j = 0; j < RBATCH; ++j) {
          ss[j] = 0.f;
#pragma unroll
          for (int v = 0; v < kHPL; ++v) ss[j] = fmaf(x1[j][v], x1[j][v], fmaf(x2[j][v], x2[j][v], ss[j]));
        }
        row_sums<LPR>(ss);
      }
#pragma unroll
      for (int j = 0; j < RBATCH; ++j) {
        const int r = b * RB + j * RPW + rsel;
        const bool isq = r < p.hq;
        if (norm) {
          const float rho = rsqrtf(ss[j] * (1.f / D) + p.eps);
          const float* w = s_w + (isq ? 0 : D);
#pragma unroll
          for (int v = 0; v < kHPL; ++v) {
            x1[j][v] = x1[j][v] * rho * w[kHPL * sub + v];
            x2[j][v] = x2[j][v] * rho * w[D / 2 + kHPL * sub + v];
          }
        }
        if (rope) {
#pragma unroll
          for (int v = 0; v < kHPL; ++v) {  // y1 = x1 c - x2 s, y2 = x2 c + x1 s
            const float a = x1[j][v], bb = x2[j][v];
            if (p.rope_bf16) {
              const float ab = bf16_round(a), bbb = bf16_round(bb);
              x1[j][v] = bf16_round(ab * c[v]) + bf16_round(-bbb * s[v]);
              x2[j][v] = bf16_round(bbb * c[v]) + bf16_round(ab * s[v]);
            } else {
              x1[j][v] = a * c[v] - bb * s[v];
              x2[j][v] = bb * c[v] + a * s[v];
            }
          }
        }
        if (r < rows) {
          const QkRows& out = isq ? p.qo : p.ko;
          const int64_t off = t * out.ts + (isq ? r : r - p.hq) * out.hs + kHPL * sub;
          store_half(out.ptr, off, true, x1[j]);
          store_half(out.ptr, off + D / 2, true, x2[j]);
        }
      }
    } else {
      const bool zero = rope && !inside;  // outside every sequence: no path to the output
      float g1[RBATCH][kHPL], g2[RBATCH][kHPL], x1[RBATCH][kHPL], x2[RBATCH][kHPL];
#pragma unroll
      for (int j = 0; j < RBATCH; ++j) {
        unstage_row(slot(st, 0, j), true, g1[j], g2[j]);
        if (norm) unstage_row(slot(st, 1, j), p.in_bf16, x1[j], x2[j]);
      }
      if (rope && !zero) {
#pragma unroll
        for (int j = 0; j < RBATCH; ++j)
#pragma unroll
          for (int v = 0; v < kHPL; ++v) {  // transpose: dn1 = g1 c + g2 s, dn2 = g2 c - g1 s
            const float a = g1[j][v], bb = g2[j][v];
            g1[j][v] = a * c[v] + bb * s[v];
            g2[j][v] = bb * c[v] - a * s[v];
          }
      }
      if (norm && !zero) {
        float ss[RBATCH], dot[RBATCH];
#pragma unroll
        for (int j = 0; j < RBATCH; ++j) {
          const bool isq = b * RB + j * RPW + rsel < p.hq;
          const float* w = s_w + (isq ? 0 : D);
          ss[j] = dot[j] = 0.f;
#pragma unroll
          for (int v = 0; v < kHPL; ++v) {
            ss[j] = fmaf(x1[j][v], x1[j][v], fmaf(x2[j][v], x2[j][v], ss[j]));
            dot[j] = fmaf(g1[j][v] * w[kHPL * sub + v], x1[j][v],
                          fmaf(g2[j][v] * w[D / 2 + kHPL * sub + v], x2[j][v], dot[j]));
          }
        }
        row_sums<LPR>(ss);
        row_sums<LPR>(dot);
#pragma unroll
        for (int j = 0; j < RBATCH; ++j) {
          const int r = b * RB + j * RPW + rsel;
          const bool isq = r < p.hq;
          const float* w = s_w + (isq ? 0 : D);
          const float rho = rsqrtf(ss[j] * (1.f / D) + p.eps);
          const float k3 = dot[j] * rho * rho * rho * (1.f / D);
#pragma unroll
          for (int v = 0; v < kHPL; ++v) {
            if (r < rows) {
              if (isq) {
                gq1[v] = fmaf(g1[j][v], x1[j][v] * rho, gq1[v]);
                gq2[v] = fmaf(g2[j][v], x2[j][v] * rho, gq2[v]);
              } else {
                gk1[v] = fmaf(g1[j][v], x1[j][v] * rho, gk1[v]);
                gk2[v] = fmaf(g2[j][v], x2[j][v] * rho, gk2[v]);
              }
            }
            g1[j][v] = g1[j][v] * w[kHPL * sub + v] * rho - x1[j][v] * k3;
            g2[j][v] = g2[j][v] * w[D / 2 + kHPL * sub + v] * rho - x2[j][v] * k3;
          }
        }
      }
#pragma unroll
      for (int j = 0; j < RBATCH; ++j) {
        const int r = b * RB + j * RPW + rsel;
        if (r >= rows) continue;
        if (zero) {
#pragma unroll
          for (int v = 0; v < kHPL; ++v) g1[j][v] = g2[j][v] = 0.f;
        }
        const bool isq = r < p.hq;
        const QkRows& gin = isq ? p.dqi : p.dki;
        const int64_t off = t * gin.ts + (isq ? r : r - p.hq) * gin.hs + kHPL * sub;
        store_half(gin.ptr, off, p.in_bf16, g1[j]);
        store_half(gin.ptr, off + D / 2, p.in_bf16, g2[j]);
      }
    }
  }
  cp_async_wait<0>();
  if (BWD && norm) {
    // weight gradients: lanes of the same column positions, warps, CTA -> one atomic per column
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1)
#pragma unroll
      for (int v = 0; v < kHPL; ++v) {
        gq1[v] += __shfl_xor_sync(0xffffffffu, gq1[v], o);
        gq2[v] += __shfl_xor_sync(0xffffffffu, gq2[v], o);
        gk1[v] += __shfl_xor_sync(0xffffffffu, gk1[v], o);
        gk2[v] += __shfl_xor_sync(0xffffffffu, gk2[v], o);
      }
    __syncthreads();  // the staging ring is reused as the reduction buffer
    float* s_dw = reinterpret_cast<float*>(prep_smem + 2 * D * 4);  // [warps][2][D]
    if (rsel == 0) {
#pragma unroll
      for (int v = 0; v < kHPL; ++v) {
        s_dw[(warp * 2 + 0) * D + kHPL * sub + v] = gq1[v];
        s_dw[(warp * 2 + 0) * D + D / 2 + kHPL * sub + v] = gq2[v];
        s_dw[(warp * 2 + 1) * D + kHPL * sub + v] = gk1[v];
        s_dw[(warp * 2 + 1) * D + D / 2 + kHPL * sub + v] = gk2[v];
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < 2 * D; e += kPrepThreads) {
      const int which = e / D, col = e % D;
      float acc = 0.f;
#pragma unroll
      for (int w8 = 0; w8 < kPrepThreads / 32; ++w8) acc += s_dw[(w8 * 2 + which) * D + col];
      atomicAdd((which ? p.dkw : p.dqw) + col, acc);
    }
  }
}

template <int D, bool BWD>
cudaError_t launch_qk_prep_t(const QkPrepParams& p, cudaStream_t stream) {
  auto kern = fna2_qk_prep_kernel<D, BWD>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(qk_prep_smem(D, 4, BWD)));
  if (e != cudaSuccess) return e;
  const size_t smem = qk_prep_smem(D, p.in_bf16 ? 2 : 4, BWD);
  int dev = 0, sms = 148, per_sm = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kPrepThreads, smem);
  if (e != cudaSuccess) return e;
  // one wave of resident CTAs, each warp at least 8 tokens
  const int64_t blocks = ((p.T + 7) / 8 + kPrepThreads / 32 - 1) / (kPrepThreads / 32);
  const int64_t wave = static_cast<int64_t>(sms) * (per_sm > 0 ? per_sm : 1);
  const int grid = static_cast<int>(blocks < wave ? (blocks > 0 ? blocks : 1) : wave);
  kern<<<grid, kPrepThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_qk_prep(const QkPrepParams& p, int D, bool bwd, cudaStream_t stream) {
  if (D == 128) return bwd ? launch_qk_prep_t<128, true>(p, stream) : launch_qk_prep_t<128, false>(p, stream);
  if (D == 64) return bwd ? launch_qk_prep_t<64, true>(p, stream) : launch_qk_prep_t<64, false>(p, stream);
  return cudaErrorInvalidValue;
}

}  // namespace fna2
