// General DC-attention forward on CUDA cores (sm_100a).
//
// This is the library's coverage kernel: it supports every composition term
// (identity, static W, query-/key-wise rank R, qdd/kdd, per-query matrix), any
// window (or full causal), seq_lens, any HPG <= 128 and D <= 128.  The tensor-
// core kernel (tc_kernel.cu) takes the windowed layers it supports; AUTO
// dispatch falls back to this one otherwise.
//
// Dataflow, one CTA per (query block of QB queries, batch b, head group g):
//   pass 0: for each key chunk of KC keys: L = scale*QK^T for all HPG heads,
//           S = compose_pre(L), masked; online row max / sum per (head, query)
//   pass 1: recompute S per chunk, P = exp(S - m) / l, P' = compose_post(P),
//           O[h, q, :] += P'[h, q, :] V_h  (fp32 accumulators in shared memory)
// The two passes are needed because the post-composition mixes the
// *normalised* probabilities of different heads (dc_attention_torch.py:236-248),
// so every head's row statistics must be final before any mixing.
// Mask after composition, NaN-free empty rows: dc_attention_torch.py:228-237.

#include <cuda_runtime.h>

#include "common.cuh"

namespace dcattn {

constexpr int KC = 32;       // keys per chunk
constexpr int NT = 256;      // threads per CTA

struct SimtGeom {
  int qb;            // queries per CTA
  size_t smem;       // dynamic shared memory bytes
};

// Shared-memory layout (all fp32 except Qs):
//   Qs  [qb][HPG][D]   (element type E)
//   Ls  [HPG][qb][KC]  logits, later probabilities
//   Ss  [HPG][qb][KC]  composed values
//   Agg [2R][qb][KC]   rank-R aggregates (query-wise r < R, key-wise r >= R)
//   Wpre, Wpost [HPG*HPG]
//   Ms, Ls_sum [HPG*qb]
//   Os  [HPG][qb][D]
inline SimtGeom simt_geom(int HPG, int D, int R, int esize) {
  SimtGeom g;
  for (g.qb = 4; g.qb > 1; g.qb /= 2) {
    size_t s = (size_t)g.qb * HPG * D * esize + 2 * (size_t)HPG * g.qb * KC * 4 +
               (size_t)2 * R * g.qb * KC * 4 + 2 * (size_t)HPG * HPG * 4 +
               2 * (size_t)HPG * g.qb * 4 + (size_t)HPG * g.qb * D * 4;
    if (s <= 200 * 1024) break;
  }
  g.smem = (size_t)g.qb * HPG * D * esize + 2 * (size_t)HPG * g.qb * KC * 4 +
           (size_t)2 * R * g.qb * KC * 4 + 2 * (size_t)HPG * HPG * 4 +
           2 * (size_t)HPG * g.qb * 4 + (size_t)HPG * g.qb * D * 4;
  g.smem = (g.smem + 15) & ~(size_t)15;
  return g;
}

// Rank-R aggregates of buffer X [HPG][qb][KC] for term set tm into Agg.
template <typename E>
__device__ void simt_aggregates(const ParamsDev &p, const TermsDev &tm, const float *X,
                                float *Agg, int qb, int b, int g, int t0, int c0,
                                int nq, int kc) {
  const int HPG = p.HPG, R = p.R, H = p.H;
  const int n = 2 * R * qb * KC;
  for (int idx = threadIdx.x; idx < n; idx += NT) {
    const int si = idx % KC, qi = (idx / KC) % qb, rr = idx / (KC * qb);
    float acc = 0.f;
    if (qi < nq && si < kc) {
      const bool keyw = rr >= R;
      const int r = keyw ? rr - R : rr;
      const void *w1 = keyw ? tm.kw1 : tm.qw1;
      if (w1) {
        const int tok = keyw ? (c0 + si) : (t0 + qi);
        const int64_t base = ((int64_t)b * p.T + tok) * H + (int64_t)g * HPG;
        for (int j = 0; j < HPG; ++j)
          acc += ldw<E>(w1, (base + j) * R + r) * X[(j * qb + qi) * KC + si];
      }
    }
    Agg[idx] = acc;
  }
}

// compose(X)[ho] at (qi, si) given precomputed aggregates.
template <typename E>
__device__ float simt_compose(const ParamsDev &p, const TermsDev &tm, const float *X,
                              const float *Agg, const float *Ws, int qb, int b, int g,
                              int ho, int qi, int si, int t, int s) {
  const int HPG = p.HPG, R = p.R, H = p.H;
  const float a = X[(ho * qb + qi) * KC + si];
  float o = tm.identity ? a : 0.f;
  if (tm.w) {
    for (int j = 0; j < HPG; ++j) o += X[(j * qb + qi) * KC + si] * Ws[j * HPG + ho];
  }
  const int hg = g * HPG + ho;
  const int64_t qtok = (int64_t)b * p.T + t, ktok = (int64_t)b * p.T + s;
  if (tm.qw2) {
    for (int r = 0; r < R; ++r)
      o += ldw<E>(tm.qw2, (qtok * R + r) * H + hg) * Agg[(r * qb + qi) * KC + si];
  }
  if (tm.kw2) {
    for (int r = 0; r < R; ++r)
      o += ldw<E>(tm.kw2, (ktok * R + r) * H + hg) * Agg[((R + r) * qb + qi) * KC + si];
  }
  float dd = 0.f;
  if (tm.qdd) dd += ldw<E>(tm.qdd, qtok * H + hg);
  if (tm.kdd) dd += ldw<E>(tm.kdd, ktok * H + hg);
  o += dd * a;
  if (tm.qmat) {
    const int64_t base = (qtok * H + hg) * HPG;
    for (int j = 0; j < HPG; ++j) o += ldw<E>(tm.qmat, base + j) * X[(j * qb + qi) * KC + si];
  }
  return o;
}

template <typename E>
__global__ void __launch_bounds__(NT) dc_simt_kernel(ParamsDev p, int qb) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int HPG = p.HPG, D = p.D, R = p.R, H = p.H;
  const int b = blockIdx.y / p.G, g = blockIdx.y % p.G;
  const int t0 = blockIdx.x * qb;
  const int nq = min(qb, p.T - t0);
  if (nq <= 0) return;

  E *Qs = reinterpret_cast<E *>(smem_raw);
  float *Ls = reinterpret_cast<float *>(smem_raw + (size_t)qb * HPG * D * sizeof(E));
  float *Ss = Ls + HPG * qb * KC;
  float *Agg = Ss + HPG * qb * KC;
  float *Wpre = Agg + 2 * R * qb * KC;
  float *Wpost = Wpre + HPG * HPG;
  float *Ms = Wpost + HPG * HPG;
  float *Lsum = Ms + HPG * qb;
  float *Os = Lsum + HPG * qb;

  const E *q = reinterpret_cast<const E *>(p.q);
  const E *k = reinterpret_cast<const E *>(p.k);
  const E *v = reinterpret_cast<const E *>(p.v);

  for (int idx = threadIdx.x; idx < qb * HPG * D; idx += NT) {
    const int d = idx % D, h = (idx / D) % HPG, qi = idx / (D * HPG);
    Qs[idx] = qi < nq ? q[(((int64_t)b * p.T + t0 + qi) * H + g * HPG + h) * D + d] : from_f<E>(0.f);
  }
  for (int idx = threadIdx.x; idx < HPG * HPG; idx += NT) {
    Wpre[idx] = p.pre.w ? p.pre.w[(int64_t)g * HPG * HPG + idx] : 0.f;
    Wpost[idx] = p.post.w ? p.post.w[(int64_t)g * HPG * HPG + idx] : 0.f;
  }
  for (int idx = threadIdx.x; idx < HPG * qb; idx += NT) {
    Ms[idx] = -INFINITY;
    Lsum[idx] = 0.f;
  }
  for (int idx = threadIdx.x; idx < HPG * qb * D; idx += NT) Os[idx] = 0.f;

  const int slen = p.seq_lens ? min(p.seq_lens[b], p.T) : p.T;
  const int kbeg = p.window > 0 ? max(0, t0 - p.window + 1) : 0;
  const int kend = min(t0 + nq, slen);
  __syncthreads();

  for (int pass = 0; pass < 2; ++pass) {
    for (int c0 = kbeg; c0 < kend; c0 += KC) {
      const int kc = min(KC, kend - c0);
      // logits
      for (int idx = threadIdx.x; idx < HPG * qb * KC; idx += NT) {
        const int si = idx % KC, qi = (idx / KC) % qb, h = idx / (KC * qb);
        float acc = 0.f;
        if (qi < nq && si < kc) {
          const E *kr = k + (((int64_t)b * p.T + c0 + si) * H + g * HPG + h) * D;
          const E *qr = Qs + (qi * HPG + h) * D;
          for (int d = 0; d < D; ++d) acc += to_f<E>(qr[d]) * to_f<E>(__ldg(kr + d));
          acc *= p.scale;
        }
        Ls[idx] = acc;
      }
      __syncthreads();
      simt_aggregates<E>(p, p.pre, Ls, Agg, qb, b, g, t0, c0, nq, kc);
      __syncthreads();
      for (int idx = threadIdx.x; idx < HPG * qb * KC; idx += NT) {
        const int si = idx % KC, qi = (idx / KC) % qb, h = idx / (KC * qb);
        const int t = t0 + qi, s = c0 + si;
        float val = -INFINITY;
        const bool valid = qi < nq && si < kc && s <= t && (p.window <= 0 || t - s < p.window);
        if (valid) val = simt_compose<E>(p, p.pre, Ls, Agg, Wpre, qb, b, g, h, qi, si, t, s);
        Ss[idx] = val;
      }
      __syncthreads();
      if (pass == 0) {
        for (int idx = threadIdx.x; idx < HPG * qb; idx += NT) {
          const float *row = Ss + idx * KC;
          float cm = -INFINITY;
          for (int si = 0; si < kc; ++si) cm = fmaxf(cm, row[si]);
          if (cm > -INFINITY) {
            const float m_old = Ms[idx];
            const float m_new = fmaxf(m_old, cm);
            float sum = Lsum[idx] * exp2f((m_old - m_new) * kLog2e);
            for (int si = 0; si < kc; ++si)
              if (row[si] > -INFINITY) sum += exp2f((row[si] - m_new) * kLog2e);
            Ms[idx] = m_new;
            Lsum[idx] = sum;
          }
        }
      } else {
        for (int idx = threadIdx.x; idx < HPG * qb * KC; idx += NT) {
          const int hq = idx / KC;
          const float sv = Ss[idx];
          const float l = Lsum[hq];
          Ls[idx] = (sv > -INFINITY && l > 0.f) ? exp2f((sv - Ms[hq]) * kLog2e) / l : 0.f;
        }
        __syncthreads();
        simt_aggregates<E>(p, p.post, Ls, Agg, qb, b, g, t0, c0, nq, kc);
        __syncthreads();
        for (int idx = threadIdx.x; idx < HPG * qb * KC; idx += NT) {
          const int si = idx % KC, qi = (idx / KC) % qb, h = idx / (KC * qb);
          float val = 0.f;
          if (qi < nq && si < kc)
            val = simt_compose<E>(p, p.post, Ls, Agg, Wpost, qb, b, g, h, qi, si, t0 + qi, c0 + si);
          Ss[idx] = val;
        }
        __syncthreads();
        for (int idx = threadIdx.x; idx < HPG * qb * D; idx += NT) {
          const int d = idx % D, hq = idx / D;  // hq = h*qb + qi
          const int h = hq / qb;
          const float *prow = Ss + hq * KC;
          const E *vcol = v + (((int64_t)b * p.T + c0) * H + g * HPG + h) * D + d;
          float acc = Os[idx];
          for (int si = 0; si < kc; ++si) acc += prow[si] * to_f<E>(__ldg(vcol + (int64_t)si * H * D));
          Os[idx] = acc;
        }
      }
      __syncthreads();
    }
  }

  E *out = reinterpret_cast<E *>(p.out);
  for (int idx = threadIdx.x; idx < HPG * qb * D; idx += NT) {
    const int d = idx % D, qi = (idx / D) % qb, h = idx / (D * qb);
    if (qi < nq)
      out[(int64_t)b * p.out_sb + (int64_t)(t0 + qi) * p.out_st + (int64_t)(g * HPG + h) * p.out_sh + d] =
          from_f<E>(Os[idx]);
  }
}

// Host launcher.  Returns cudaError_t of the launch.
template <typename E>
static cudaError_t launch_simt_t(const ParamsDev &p, cudaStream_t st) {
  SimtGeom gm = simt_geom(p.HPG, p.D, p.R, (int)sizeof(E));
  cudaError_t e = cudaFuncSetAttribute(dc_simt_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)gm.smem);
  if (e != cudaSuccess) return e;
  dim3 grid((p.T + gm.qb - 1) / gm.qb, p.B * p.G);
  dc_simt_kernel<E><<<grid, NT, gm.smem, st>>>(p, gm.qb);
  return cudaGetLastError();
}

cudaError_t launch_simt(const ParamsDev &p, int dtype, cudaStream_t st) {
  if (dtype == DC_DTYPE_BF16) return launch_simt_t<__nv_bfloat16>(p, st);
  return launch_simt_t<__half>(p, st);
}

size_t simt_smem_bytes(int HPG, int D, int R, int dtype) {
  (void)dtype;
  return simt_geom(HPG, D, R, 2).smem;
}

}  // namespace dcattn
