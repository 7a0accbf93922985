// Varlen QK-RMSNorm + RoPE pre-attention transform (forward and backward).
//
// Reference semantics: FNA2/attention_fna2.py RMSNorm.forward (:100-102):
// n = x * rsqrt(mean(x^2) + eps) * w; RotaryPositionalEmbedding (:108-163):
// y = n*cos + rotate_half(n)*sin with cos/sin = cos/sin(cat(t*f, t*f)), the
// table built in the dtype of the rotated tensor (:148-155); and
// _apply_rope_varlen (:620-647): t restarts at 0 for every packed sequence.
//
// HBM-bound elementwise work: one warp handles one row (token, head) of
// head_dim values, head_dim/32 per lane; the rotate_half partner of lane l is
// lane l^16.  A CTA owns a block of consecutive tokens; the tokens' positions
// come from one binary search over cu_seqlens per token (shared by all heads
// of that token) and the cos/sin values of a token are computed once per warp
// and reused for every head.  The backward recomputes the norm and
// accumulates the weight gradients per warp, then per CTA, then with one
// atomic per column and CTA (grid-stride, a few CTAs per SM).
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
constexpr int kRowBatch = 4;    // row instructions whose loads a warp issues together (forward)
constexpr int kRowBatchBwd = 2;  // the same for the backward (twice the operands per row)

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// A row (one token, one head, D values) is spread over LPR = D/8 lanes, 8
// consecutive values per lane (one 16-byte bf16 access), so a warp covers
// RPW = 32/LPR rows per instruction; the rotate_half partner of a lane is
// lane ^ (LPR/2) and row sums reduce over the LPR lanes of a row.
constexpr int kEPL = 8;

__device__ __forceinline__ void load8(const void* base, int64_t off, bool is_bf16, bool valid, float (&x)[kEPL]) {
  if (!valid) {
#pragma unroll
    for (int u = 0; u < kEPL; ++u) x[u] = 0.f;
    return;
  }
  if (is_bf16) {
    const uint4 w = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(base) + off);
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ww[i]));
      x[2 * i] = f.x, x[2 * i + 1] = f.y;
    }
  } else {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + off);
    const float4 a = p[0], b = p[1];
    x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
  }
}

__device__ __forceinline__ void store8(void* base, int64_t off, bool is_bf16, const float (&y)[kEPL]) {
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

// cos/sin of this lane's 8 columns at position pos, formed as the reference
// forms its table: fp32 t*f, or (bf16 mode) t, f and t*f rounded to bf16 and
// cos/sin rounded to bf16.
template <int D>
__device__ __forceinline__ void rope_table(const QkPrepParams& p, int pos, int sub, float (&c)[kEPL],
                                           float (&s)[kEPL]) {
#pragma unroll
  for (int u = 0; u < kEPL; ++u) {
    const int i = (kEPL * sub + u) % (D / 2);
    const float f = __ldg(p.inv_freq + i), t = static_cast<float>(pos);
    const float ang = p.rope_bf16 ? bf16_round(bf16_round(t) * bf16_round(f)) : t * f;
    sincosf(ang, &s[u], &c[u]);
    if (p.rope_bf16) {
      c[u] = bf16_round(c[u]);
      s[u] = bf16_round(s[u]);
    }
  }
}

__device__ __forceinline__ void load_weight8(const void* w, bool is_bf16, int sub, float (&wv)[kEPL]) {
#pragma unroll
  for (int u = 0; u < kEPL; ++u) {
    const int e = kEPL * sub + u;
    wv[u] = is_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(w)[e]) : static_cast<const float*>(w)[e];
  }
}

template <int LPR>
__device__ __forceinline__ float row_sum(float v) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Per-warp walk over a contiguous run of tokens; calls body(t, pos, valid_rope)
// with the token's position within its sequence (consecutive tokens mostly
// share the sequence bounds found last).
template <typename F>
__device__ __forceinline__ void for_each_token(const QkPrepParams& p, bool rope, int lane, F&& body) {
  const int64_t nw = static_cast<int64_t>(gridDim.x) * (kPrepThreads / 32);
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * (kPrepThreads / 32) + (threadIdx.x >> 5);
  const int64_t chunk = (p.T + nw - 1) / nw;
  const int64_t t_end = min(p.T, (gw + 1) * chunk);
  int s_lo = 0, s_hi = 0;
  for (int64_t t = gw * chunk; t < t_end; ++t) {
    bool inside = true;
    if (rope && (t < s_lo || t >= s_hi)) {
      inside = warp_find_sequence(p, t, lane, &s_lo, &s_hi);
      if (!inside) s_lo = s_hi = 0;
    }
    body(t, inside ? static_cast<int>(t - s_lo) : 0, inside);
  }
}

template <int D>
__global__ void __launch_bounds__(kPrepThreads) fna2_qk_prep_fwd_kernel(const QkPrepParams p) {
  constexpr int LPR = D / kEPL, RPW = 32 / LPR;
  const int lane = threadIdx.x & 31, sub = lane % LPR, rsel = lane / LPR;
  const bool rope = p.inv_freq != nullptr;
  const int rows = p.hq + p.hk;
  float wq[kEPL], wk[kEPL];
  if (p.qw) load_weight8(p.qw, p.w_bf16, sub, wq);
  if (p.kw) load_weight8(p.kw, p.w_bf16, sub, wk);
  const float sign = sub < LPR / 2 ? -1.f : 1.f;  // rotate_half: [-x2, x1]
  for_each_token(p, rope, lane, [&](int64_t t, int pos, bool inside) {
    if (rope && !inside) return;  // outside every sequence: left unset, as the reference does
    float c[kEPL], s[kEPL];
    if (rope) rope_table<D>(p, pos, sub, c, s);
    for (int r0 = 0; r0 < rows; r0 += kRowBatch * RPW) {
      float x[kRowBatch][kEPL], ss[kRowBatch];
#pragma unroll
      for (int j = 0; j < kRowBatch; ++j) {  // loads of the whole batch first
        const int r = r0 + j * RPW + rsel;
        const bool isq = r < p.hq;
        const QkRows& in = isq ? p.qi : p.ki;
        load8(in.ptr, t * in.ts + (isq ? r : r - p.hq) * in.hs + kEPL * sub, p.in_bf16, r < rows, x[j]);
      }
      if (p.qw) {
#pragma unroll
        for (int j = 0; j < kRowBatch; ++j) {
          ss[j] = 0.f;
#pragma unroll
          for (int u = 0; u < kEPL; ++u) ss[j] = fmaf(x[j][u], x[j][u], ss[j]);
        }
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1)
#pragma unroll
          for (int j = 0; j < kRowBatch; ++j) ss[j] += __shfl_xor_sync(0xffffffffu, ss[j], o);
      }
#pragma unroll
      for (int j = 0; j < kRowBatch; ++j) {
        const int r = r0 + j * RPW + rsel;
        const bool isq = r < p.hq;
        if (p.qw) {
          const float rho = rsqrtf(ss[j] * (1.f / D) + p.eps);
#pragma unroll
          for (int u = 0; u < kEPL; ++u) x[j][u] = x[j][u] * rho * (isq ? wq[u] : wk[u]);
        }
        if (rope) {
#pragma unroll
          for (int u = 0; u < kEPL; ++u) {
            const float partner = __shfl_xor_sync(0xffffffffu, x[j][u], LPR / 2);
            if (p.rope_bf16) {
              const float xb = bf16_round(x[j][u]), pb = bf16_round(partner);
              x[j][u] = bf16_round(xb * c[u]) + bf16_round(sign * pb * s[u]);
            } else {
              x[j][u] = x[j][u] * c[u] + sign * partner * s[u];
            }
          }
        }
        if (r < rows) {
          const QkRows& out = isq ? p.qo : p.ko;
          store8(out.ptr, t * out.ts + (isq ? r : r - p.hq) * out.hs + kEPL * sub, true, x[j]);
        }
      }
    }
  });
}

template <int D>
__global__ void __launch_bounds__(kPrepThreads) fna2_qk_prep_bwd_kernel(const QkPrepParams p) {
  constexpr int LPR = D / kEPL, RPW = 32 / LPR;
  __shared__ float s_dw[2][kPrepThreads / 32][D];
  const int lane = threadIdx.x & 31, sub = lane % LPR, rsel = lane / LPR;
  const bool rope = p.inv_freq != nullptr;
  const bool norm = p.qw != nullptr;
  const int rows = p.hq + p.hk;
  float wq[kEPL], wk[kEPL], gq[kEPL], gk[kEPL];
#pragma unroll
  for (int u = 0; u < kEPL; ++u) gq[u] = gk[u] = 0.f;
  if (norm) {
    load_weight8(p.qw, p.w_bf16, sub, wq);
    load_weight8(p.kw, p.w_bf16, sub, wk);
  }
  const float sign = sub < LPR / 2 ? 1.f : -1.f;  // rotate_half^T(v) = [v[D/2:], -v[:D/2]]
  for_each_token(p, rope, lane, [&](int64_t t, int pos, bool inside) {
    if (rope && !inside) {  // outside every sequence: no path to the output
      float z[kEPL];
#pragma unroll
      for (int u = 0; u < kEPL; ++u) z[u] = 0.f;
      for (int r = rsel; r < rows; r += RPW) {
        const bool isq = r < p.hq;
        const QkRows& gin = isq ? p.dqi : p.dki;
        store8(gin.ptr, t * gin.ts + (isq ? r : r - p.hq) * gin.hs + kEPL * sub, p.in_bf16, z);
      }
      return;
    }
    float c[kEPL], s[kEPL];
    if (rope) rope_table<D>(p, pos, sub, c, s);
    for (int r0 = 0; r0 < rows; r0 += kRowBatchBwd * RPW) {
      float g[kRowBatchBwd][kEPL], x[kRowBatchBwd][kEPL];
#pragma unroll
      for (int j = 0; j < kRowBatchBwd; ++j) {
        const int r = r0 + j * RPW + rsel;
        const bool isq = r < p.hq;
        const int hh = isq ? r : r - p.hq;
        const QkRows& gout = isq ? p.dqo : p.dko;
        load8(gout.ptr, t * gout.ts + hh * gout.hs + kEPL * sub, true, r < rows, g[j]);
        if (norm) {
          const QkRows& in = isq ? p.qi : p.ki;
          load8(in.ptr, t * in.ts + hh * in.hs + kEPL * sub, p.in_bf16, r < rows, x[j]);
        }
      }
      if (rope) {
        // transpose of the rotation: dn = dy*cos + rotate_half^T(dy)*sin
#pragma unroll
        for (int j = 0; j < kRowBatchBwd; ++j)
#pragma unroll
          for (int u = 0; u < kEPL; ++u) {
            const float partner = __shfl_xor_sync(0xffffffffu, g[j][u], LPR / 2);
            g[j][u] = g[j][u] * c[u] + sign * partner * s[u];
          }
      }
      if (norm) {
        float ss[kRowBatchBwd], dot[kRowBatchBwd];
#pragma unroll
        for (int j = 0; j < kRowBatchBwd; ++j) {
          const bool isq = r0 + j * RPW + rsel < p.hq;
          ss[j] = dot[j] = 0.f;
#pragma unroll
          for (int u = 0; u < kEPL; ++u) {
            ss[j] = fmaf(x[j][u], x[j][u], ss[j]);
            dot[j] = fmaf(g[j][u] * (isq ? wq[u] : wk[u]), x[j][u], dot[j]);
          }
        }
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1)
#pragma unroll
          for (int j = 0; j < kRowBatchBwd; ++j) {
            ss[j] += __shfl_xor_sync(0xffffffffu, ss[j], o);
            dot[j] += __shfl_xor_sync(0xffffffffu, dot[j], o);
          }
#pragma unroll
        for (int j = 0; j < kRowBatchBwd; ++j) {
          const int r = r0 + j * RPW + rsel;
          const bool isq = r < p.hq;
          const float rho = rsqrtf(ss[j] * (1.f / D) + p.eps);
          const float k3 = dot[j] * rho * rho * rho * (1.f / D);
#pragma unroll
          for (int u = 0; u < kEPL; ++u) {
            if (r < rows) {
              if (isq) gq[u] = fmaf(g[j][u], x[j][u] * rho, gq[u]);
              else gk[u] = fmaf(g[j][u], x[j][u] * rho, gk[u]);
            }
            g[j][u] = g[j][u] * (isq ? wq[u] : wk[u]) * rho - x[j][u] * k3;
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kRowBatchBwd; ++j) {
        const int r = r0 + j * RPW + rsel;
        if (r >= rows) continue;
        const bool isq = r < p.hq;
        const QkRows& gin = isq ? p.dqi : p.dki;
        store8(gin.ptr, t * gin.ts + (isq ? r : r - p.hq) * gin.hs + kEPL * sub, p.in_bf16, g[j]);
      }
    }
  });
  if (norm) {
    // weight gradients: the lanes of a row position, warps, CTA -> one atomic per column
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1)
#pragma unroll
      for (int u = 0; u < kEPL; ++u) {
        gq[u] += __shfl_xor_sync(0xffffffffu, gq[u], o);
        gk[u] += __shfl_xor_sync(0xffffffffu, gk[u], o);
      }
    const int warp = threadIdx.x >> 5;
    if (rsel == 0) {
#pragma unroll
      for (int u = 0; u < kEPL; ++u) {
        s_dw[0][warp][kEPL * sub + u] = gq[u];
        s_dw[1][warp][kEPL * sub + u] = gk[u];
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < 2 * D; e += kPrepThreads) {
      const int which = e / D, col = e % D;
      float acc = 0.f;
#pragma unroll
      for (int w8 = 0; w8 < kPrepThreads / 32; ++w8) acc += s_dw[which][w8][col];
      atomicAdd((which ? p.dkw : p.dqw) + col, acc);
    }
  }
}

inline int qk_prep_grid(int64_t T) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t warps = (T + 7) / 8;  // at least 8 tokens per warp
  const int64_t blocks = (warps + kPrepThreads / 32 - 1) / (kPrepThreads / 32);
  return static_cast<int>(blocks < 8LL * sms ? (blocks > 0 ? blocks : 1) : 8LL * sms);
}

cudaError_t launch_qk_prep(const QkPrepParams& p, int D, bool bwd, cudaStream_t stream) {
  const int grid = qk_prep_grid(p.T);
  if (D == 128) {
    if (bwd) fna2_qk_prep_bwd_kernel<128><<<grid, kPrepThreads, 0, stream>>>(p);
    else fna2_qk_prep_fwd_kernel<128><<<grid, kPrepThreads, 0, stream>>>(p);
  } else if (D == 64) {
    if (bwd) fna2_qk_prep_bwd_kernel<64><<<grid, kPrepThreads, 0, stream>>>(p);
    else fna2_qk_prep_fwd_kernel<64><<<grid, kPrepThreads, 0, stream>>>(p);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace fna2
