// Two-pass streaming tensor-core DC-attention forward for 32 heads per group
// (G = 1 at H = 32: every head mixes with every other) on sm_100a.
//
// Same dataflow as tcs_kernel.cu (pass A: running softmax statistics of the
// composed logits; pass B: normalise, post-compose, P'V), but a block of 8
// queries x 32 heads = 256 (head, query) columns: with 16 queries the S tile
// alone would fill all 512 TMEM columns.  N = 8 needs M = 64 tcgen05 MMAs:
//   QK  per head, two 64-key sub-tiles; sub-tile u writes TMEM lanes
//       16u + 32q + r (r < 16) of every lane quarter q, so thread (quarter q,
//       lane l) holds key 64 (l / 16) + 16 q + (l % 16) of the 128-key tile;
//   PV  per head, the two 64-d halves of V^T the same way: thread (q, l)
//       accumulates d = 64 (l / 16) + 16 q + (l % 16).
// Composition of the 32 heads is thread-local as in the other kernels; the
// 32 x 32 static mix runs on CUDA cores from shared memory (broadcast float4
// loads), the per-key weights stream from L1 in 8-head chunks, and a compose
// group is 2 queries x 32 heads (64 values).

#include <cuda.h>
#include <cuda_runtime.h>

#include <string>
#include <type_traits>

#include "tc_common.cuh"

namespace dcattn {
namespace tcs32 {

using namespace tc;

constexpr int HPG = 32, BM = 8, NQT = 256, NCW = 8, NSLOT = 2;
constexpr int QPG = 2;                 // queries per compose group
constexpr int NGRP = BM / QPG;         // 4 groups per key, 2 per compose warp

struct GeoS32 {
  int q_off, ring_off, p_off, wz_off, rec_off, red_off, stat_off, bar_off, tmem_off, total, rec_floats;
};

template <int R>
__host__ __device__ inline GeoS32 make_geo_32() {
  GeoS32 g{};
  g.q_off = 0;                                   // 32 heads x 8 queries x 256 B = 64 KB (later: output staging)
  g.ring_off = NQT * 256;
  g.p_off = g.ring_off + NSLOT * TILE_BYTES;     // P': 32 heads x 128 keys x 8 queries x 2 B = 64 KB
  int o = g.p_off + KT_ROWS * NQT * 2;
  g.rec_floats = round_up(HPG * (2 * R + 1), 4);
  g.wz_off = o; o += 2 * HPG * HPG * 4;
  g.rec_off = round_up(o, 16); o = g.rec_off + 2 * BM * g.rec_floats * 4;
  g.red_off = o; o += 2 * 4 * NQT * 4;
  g.stat_off = o; o += 2 * NQT * 4;
  g.bar_off = round_up(o, 8); o = g.bar_off + 24 * 8;
  g.tmem_off = o; o += 16;
  g.total = o;
  return g;
}

// 8 consecutive per-key weights (bf16/fp16) as floats, through L1.
template <typename E>
__device__ __forceinline__ void ld8(const void *base, int64_t idx, float (&w)[8]) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(reinterpret_cast<const E *>(base) + idx));
  const E *e = reinterpret_cast<const E *>(&raw);
#pragma unroll
  for (int j = 0; j < 8; ++j) w[j] = to_f<E>(e[j]);
}

// Composition of two queries (same key) across the 32 heads.  Wt: static mix
// (transposed, zero diagonal, shared memory); rec0/rec1: per-query records
// (dq | qa | qb); kw*: the key's per-key weights in global memory (token tok),
// absent terms NULL.
template <typename E, int R>
__device__ __forceinline__ void compose32x2(const float (&a0)[HPG], const float (&a1)[HPG], float (&o0)[HPG],
                                            float (&o1)[HPG], const float *Wt, const float *rec0,
                                            const float *rec1, const TermPtrs &tm, int64_t tok, int H,
                                            int hbase, bool key_ok) {
  const float *dq0 = rec0, *qa0 = rec0 + HPG, *qb0 = rec0 + HPG + HPG * R;
  const float *dq1 = rec1, *qa1 = rec1 + HPG, *qb1 = rec1 + HPG + HPG * R;
  float aq0[R], aq1[R], ak0[R], ak1[R];
#pragma unroll
  for (int r = 0; r < R; ++r) { aq0[r] = aq1[r] = ak0[r] = ak1[r] = 0.f; }
#pragma unroll
  for (int h = 0; h < HPG; ++h)
#pragma unroll
    for (int r = 0; r < R; ++r) {
      aq0[r] = fmaf(qa0[h * R + r], a0[h], aq0[r]);
      aq1[r] = fmaf(qa1[h * R + r], a1[h], aq1[r]);
    }
  const bool has_k1 = key_ok && tm.kw1, has_dd = key_ok && tm.kdd;
  if (has_k1) {
#pragma unroll
    for (int c = 0; c < HPG * R; c += 8) {
      float w[8];
      ld8<E>(tm.kw1, (tok * H + hbase) * R + c, w);  // kw1[tok, hbase + h, r], flat index h*R + r
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int h = (c + j) / R, r = (c + j) % R;
        ak0[r] = fmaf(w[j], a0[h], ak0[r]);
        ak1[r] = fmaf(w[j], a1[h], ak1[r]);
      }
    }
  }
#pragma unroll
  for (int c = 0; c < HPG; c += 8) {
    float kd[8], k2[R][8];
    if (has_dd) {
      ld8<E>(tm.kdd, tok * H + hbase + c, kd);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) kd[j] = 0.f;
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (has_k1) {
        ld8<E>(tm.kw2, (tok * R + r) * H + hbase + c, k2[r]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) k2[r][j] = 0.f;
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int h = c + j;
      float x0 = (dq0[h] + kd[j]) * a0[h], x1 = (dq1[h] + kd[j]) * a1[h];
#pragma unroll
      for (int hp = 0; hp < HPG; hp += 4) {
        const float4 w = *reinterpret_cast<const float4 *>(Wt + h * HPG + hp);
        x0 = fmaf(w.x, a0[hp], fmaf(w.y, a0[hp + 1], fmaf(w.z, a0[hp + 2], fmaf(w.w, a0[hp + 3], x0))));
        x1 = fmaf(w.x, a1[hp], fmaf(w.y, a1[hp + 1], fmaf(w.z, a1[hp + 2], fmaf(w.w, a1[hp + 3], x1))));
      }
#pragma unroll
      for (int r = 0; r < R; ++r) {
        x0 = fmaf(qb0[r * HPG + h], aq0[r], fmaf(k2[r][j], ak0[r], x0));
        x1 = fmaf(qb1[r * HPG + h], aq1[r], fmaf(k2[r][j], ak1[r], x1));
      }
      o0[h] = x0;
      o1[h] = x1;
    }
  }
}

template <typename E, int R>
__global__ void __launch_bounds__(32 * (NCW + 2), 1)
    dc_tcs32_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                    const TcParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                          ~static_cast<uintptr_t>(1023));
  const GeoS32 geo = make_geo_32<R>();
  float *Wz = reinterpret_cast<float *>(smem + geo.wz_off);
  float *rec = reinterpret_cast<float *>(smem + geo.rec_off);
  float *redm = reinterpret_cast<float *>(smem + geo.red_off), *reds = redm + 4 * NQT;
  float *mval = reinterpret_cast<float *>(smem + geo.stat_off), *linv = mval + NQT;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + geo.bar_off);
  uint64_t *bar_full = bars + 0, *bar_free = bars + 3, *bar_q = bars + 6;
  uint64_t *bar_S = bars + 7, *bar_Sfree = bars + 8, *bar_P = bars + 9, *bar_Pfree = bars + 10;
  uint64_t *bar_O = bars + 11;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + geo.tmem_off);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tma_warp = NCW, mma_warp = NCW + 1;
  const int nqb = (p.T + BM - 1) / BM;
  const int qb = nqb - 1 - static_cast<int>(blockIdx.x);
  const int b = blockIdx.y / p.G, g = blockIdx.y % p.G;
  const int q0 = qb * BM, H = p.H, T = p.T, hbase = g * HPG;
  const int k_lo = p.window > 0 ? max(0, q0 - p.window + 1) : 0;
  const int span = min(q0 + BM, T) - k_lo;
  const int nkt = (span + KT_ROWS - 1) / KT_ROWS;
  const int rlast = ((span - KT_ROWS * (nkt - 1)) + 15) / 16 * 16;
  const int slen = p.seq_lens ? min(max(p.seq_lens[b], 0), T) : T;
  const uint32_t WAIT = 1u << 24;
  const uint32_t o_col = NQT;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 3; ++i) {
      ptx::mbar_init(bar_full + i, 1);
      ptx::mbar_init(bar_free + i, 1);
    }
    ptx::mbar_init(bar_q, 1);
    ptx::mbar_init(bar_S, 1);
    ptx::mbar_init(bar_Sfree, NCW);
    ptx::mbar_init(bar_P, NCW);
    ptx::mbar_init(bar_Pfree, 1);
    ptx::mbar_init(bar_O, 1);
    ptx::fence_mbar_init();
  }
  if (warp == tma_warp) ptx::tmem_alloc(tmem_slot, 512);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == tma_warp) {
    // ================================================= TMA producer (job order as in tcs_kernel.cu)
    if (lane == 0) {
      ptx::tma_prefetch_desc(&tm_q);
      ptx::tma_prefetch_desc(&tm_k);
      ptx::tma_prefetch_desc(&tm_v);
      ptx::mbar_expect_tx(bar_q, NQT * 256);
      for (int h = 0; h < HPG; ++h)
        for (int c = 0; c < 2; ++c)
          ptx::tma_load_4d(smem + geo.q_off + h * BM * 256 + c * BM * 128, &tm_q, bar_q, c * 64, hbase + h, q0, b);
      int job = 0;
      bool ok = true;
      auto load = [&](const CUtensorMap *m, int kt, int h) {
        if (!ok) return;
        const int slot = job % NSLOT, use = job / NSLOT;
        if (use > 0 && !ptx::mbar_wait(bar_free + slot, (use - 1) & 1, WAIT)) {
          ok = false;
          record_err(p, ERR_TIMEOUT_FREE);
          return;
        }
        ptx::mbar_expect_tx(bar_full + slot, TILE_BYTES);
        unsigned char *dst = smem + geo.ring_off + slot * TILE_BYTES;
        ptx::tma_load_4d(dst, m, bar_full + slot, 0, hbase + h, k_lo + kt * KT_ROWS, b);
        ptx::tma_load_4d(dst + TILE_BYTES / 2, m, bar_full + slot, 64, hbase + h, k_lo + kt * KT_ROWS, b);
        ++job;
      };
      for (int kt = 0; kt < nkt; ++kt)
        for (int h = 0; h < HPG; ++h) load(&tm_k, kt, h);
      for (int kt = 0; kt < nkt; ++kt) {
        for (int h = 0; h < HPG; ++h) load(&tm_k, kt, h);
        if (kt >= 1)
          for (int h = 0; h < HPG; ++h) load(&tm_v, kt - 1, h);
      }
      for (int h = 0; h < HPG; ++h) load(&tm_v, nkt - 1, h);
    }
    __syncwarp();
  } else if (warp == mma_warp) {
    // ================================================= MMA issuer (M = 64, N = 8)
    if (lane == 0) {
      const uint32_t ab_fmt = std::is_same<E, __nv_bfloat16>::value ? 1u : 0u;
      const uint32_t idesc_qk = ptx::idesc_f16(ab_fmt, 0, 0, 64, BM);
      const uint32_t idesc_pv = ptx::idesc_f16(ab_fmt, 1, 1, 64, BM);
      const uint32_t q_addr = ptx::smem_u32(smem + geo.q_off);
      const uint32_t ring_addr = ptx::smem_u32(smem + geo.ring_off);
      const uint32_t p_addr = ptx::smem_u32(smem + geo.p_off);
      int job = 0;
      bool ok = ptx::mbar_wait(bar_q, 0, WAIT);
      if (!ok) record_err(p, ERR_TIMEOUT_Q);
      ptx::tc_fence_after();
      auto qk = [&](int sidx) {
        if (sidx >= 1 && !ptx::mbar_wait(bar_Sfree, (sidx - 1) & 1, WAIT)) {
          ok = false;
          record_err(p, ERR_TIMEOUT_S);
          return;
        }
        ptx::tc_fence_after();
        for (int h = 0; h < HPG && ok; ++h, ++job) {
          const int slot = job % NSLOT;
          if (!ptx::mbar_wait(bar_full + slot, (job / NSLOT) & 1, WAIT)) {
            ok = false;
            record_err(p, ERR_TIMEOUT_FULL);
            return;
          }
          ptx::tc_fence_after();
          const uint32_t a0 = ring_addr + slot * TILE_BYTES;
          const uint32_t b0 = q_addr + h * BM * 256;
#pragma unroll
          for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
              // 64-key sub-tile u: rows 64u.. of the K tile (64 rows x 128 B = 8 KB per d half)
              const uint64_t ad =
                  ptx::smem_desc(a0 + u * 8192 + (ks >> 2) * (TILE_BYTES / 2) + (ks & 3) * 32, 16, 1024, 2);
              const uint64_t bd = ptx::smem_desc(b0 + (ks >> 2) * (BM * 128) + (ks & 3) * 32, 16, 1024, 2);
              ptx::mma_f16_ss(tbase + (static_cast<uint32_t>(16 * u) << 16) + h * BM, ad, bd, idesc_qk, ks > 0);
            }
          ptx::mma_commit(bar_free + slot);
        }
        ptx::mma_commit(bar_S);
      };
      auto pv = [&](int kt) {
        if (!ptx::mbar_wait(bar_P, kt & 1, WAIT)) {
          ok = false;
          record_err(p, ERR_TIMEOUT_P);
          return;
        }
        ptx::tc_fence_after();
        const int rows = kt == nkt - 1 ? rlast : KT_ROWS;
        for (int h = 0; h < HPG && ok; ++h, ++job) {
          const int slot = job % NSLOT;
          if (!ptx::mbar_wait(bar_full + slot, (job / NSLOT) & 1, WAIT)) {
            ok = false;
            record_err(p, ERR_TIMEOUT_FULL);
            return;
          }
          ptx::tc_fence_after();
          const uint32_t a0 = ring_addr + slot * TILE_BYTES;
          const uint32_t b0 = p_addr + h * (KT_ROWS * BM * 2);
#pragma unroll
          for (int c = 0; c < 2; ++c)
            for (int ks = 0; ks < rows / 16; ++ks) {
              // d half c of V^T: MN-major 128B swizzle, one 64-wide M block
              const uint64_t ad = ptx::smem_desc(a0 + c * (TILE_BYTES / 2) + ks * 2048, TILE_BYTES / 2, 1024, 2);
              const uint64_t bd = ptx::smem_desc(b0 + ks * (2 * BM * 16), BM * 16, 128, 0);
              ptx::mma_f16_ss(tbase + (static_cast<uint32_t>(16 * c) << 16) + o_col + h * BM, ad, bd, idesc_pv,
                              (kt > 0 || ks > 0));
            }
          ptx::mma_commit(bar_free + slot);
        }
        ptx::mma_commit(bar_Pfree);
      };
      for (int kt = 0; kt < nkt && ok; ++kt) qk(kt);
      for (int kt = 0; kt < nkt && ok; ++kt) {
        qk(nkt + kt);
        if (kt >= 1 && ok) pv(kt - 1);
      }
      if (ok) pv(nkt - 1);
      ptx::mma_commit(bar_O);
    }
    __syncwarp();
  } else {
    // ================================================= compose warps
    const int sub = warp & 3, cs = warp >> 2;
    const int key_local = 64 * (lane >> 4) + 16 * sub + (lane & 15);  // key of this lane in a tile
    const int ctid = threadIdx.x;
    const float sl2e = p.scale * kLog2e;
    // value index L (0..63) of a group <-> (head L / 2, query i0 + L % 2)
    auto col_of = [&](int L, int i0) { return (L >> 1) * BM + i0 + (L & 1); };

    for (int idx = ctid; idx < 2 * HPG * HPG; idx += 32 * NCW) {
      const int set = idx / (HPG * HPG), j = idx % (HPG * HPG);
      const TermPtrs &tm = set ? p.post : p.pre;
      const int h = j / HPG, hp = j % HPG;
      Wz[idx] = (hp == h || !tm.w) ? 0.f : tm.w[((int64_t)g * HPG + hp) * HPG + h];
    }
    for (int idx = ctid; idx < 2 * BM * geo.rec_floats; idx += 32 * NCW) {
      const int set = idx / (BM * geo.rec_floats), rem = idx % (BM * geo.rec_floats);
      const int i = rem / geo.rec_floats, j = rem % geo.rec_floats;
      const TermPtrs &tm = set ? p.post : p.pre;
      const int t = q0 + i;
      float val = 0.f;
      if (t < T) {
        const int64_t tok = (int64_t)b * T + t;
        if (j < HPG) {
          val = (tm.identity ? 1.f : 0.f) + (tm.w ? tm.w[((int64_t)g * HPG + j) * HPG + j] : 0.f) +
                (tm.qdd ? ld_w<E>(tm.qdd, tok * H + hbase + j) : 0.f);
        } else if (j < HPG + HPG * R) {
          const int h = (j - HPG) / R, r = (j - HPG) % R;
          val = tm.qw1 ? ld_w<E>(tm.qw1, (tok * H + hbase + h) * R + r) : 0.f;
        } else if (j < HPG + 2 * HPG * R) {
          const int r = (j - HPG - HPG * R) / HPG, h = (j - HPG - HPG * R) % HPG;
          val = tm.qw2 ? ld_w<E>(tm.qw2, (tok * R + r) * H + hbase + h) : 0.f;
        }
      }
      rec[idx] = val;
    }
    ptx::named_bar_sync(1, 32 * NCW);

    // running statistics: 2 groups x 2 blocks of 32 values per compose warp
    float m_run[4], l_run[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) { m_run[k] = -INFINITY; l_run[k] = 0.f; }
    bool ok = true;
    const uint32_t tl = tbase + (static_cast<uint32_t>(32 * sub) << 16);

    // one 64-value group: S (TMEM) -> composed, masked logits in v0 / v1
    auto compose_pre = [&](int i0, int s, bool key_ok, float (&v0)[HPG], float (&v1)[HPG]) {
      float a0[HPG], a1[HPG];
#pragma unroll
      for (int h = 0; h < HPG; ++h) {
        float x[2];
        ptx::tmem_ld<2>(tl + h * BM + i0, x);
        a0[h] = x[0];
        a1[h] = x[1];
      }
      ptx::tmem_wait_ld();
      compose32x2<E, R>(a0, a1, v0, v1, Wz, rec + i0 * geo.rec_floats, rec + (i0 + 1) * geo.rec_floats, p.pre,
                        (int64_t)b * T + s, H, hbase, key_ok);
      const int t0 = q0 + i0, t1 = t0 + 1;
      const bool ok0 = key_ok && s <= t0 && (p.window <= 0 || t0 - s < p.window) && t0 < T;
      const bool ok1 = key_ok && s <= t1 && (p.window <= 0 || t1 - s < p.window) && t1 < T;
#pragma unroll
      for (int h = 0; h < HPG; ++h) {
        v0[h] = ok0 ? v0[h] : -INFINITY;
        v1[h] = ok1 ? v1[h] : -INFINITY;
      }
    };

    // ---- pass A
    for (int kt = 0; kt < nkt; ++kt) {
      const int s = k_lo + kt * KT_ROWS + key_local;
      const int rows = kt == nkt - 1 ? rlast : KT_ROWS;
      const bool key_ok = s < slen && key_local < rows;
      const bool active = __any_sync(0xffffffffu, key_ok && s <= q0 + BM - 1 &&
                                                      (p.window <= 0 || s >= q0 - p.window + 1));
      if (ok && !ptx::mbar_wait(bar_S, kt & 1, WAIT)) { ok = false; record_err(p, ERR_TIMEOUT_S); }
      ptx::tc_fence_after();
#pragma unroll 1
      for (int k = 0; k < NGRP / 2; ++k) {
        const int i0 = (cs * (NGRP / 2) + k) * QPG;
        if (!(active && ok)) continue;
        float v0[HPG], v1[HPG];
        compose_pre(i0, s, key_ok, v0, v1);
        // two blocks of 32 values: block 0 = heads 0..15, block 1 = heads 16..31 (x 2 queries)
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
          float x[32], mt = -INFINITY;
#pragma unroll
          for (int L = 0; L < 32; ++L) {
            const int h = 16 * blk + (L >> 1);
            const float val = (L & 1) ? v1[h] : v0[h];
            const float mw = ptx::warp_max(val);
            if (lane == L) mt = mw;
            x[L] = exp2f((val - (mw == -INFINITY ? 0.f : mw)) * sl2e);
          }
#pragma unroll
          for (int off = 16, cnt = 32; off >= 1; off >>= 1, cnt >>= 1) {
            const bool upper = (lane & off) != 0;
#pragma unroll
            for (int j = 0; j < cnt / 2; ++j) {
              const float send = upper ? x[j] : x[j + cnt / 2];
              const float keep = upper ? x[j + cnt / 2] : x[j];
              x[j] = keep + __shfl_xor_sync(0xffffffffu, send, off);
            }
          }
          const int rk = 2 * k + blk;
          if (mt != -INFINITY) {
            const float mn = fmaxf(m_run[rk], mt);
            l_run[rk] = (m_run[rk] == -INFINITY ? 0.f : l_run[rk] * exp2f((m_run[rk] - mn) * sl2e)) +
                        x[0] * exp2f((mt - mn) * sl2e);
            m_run[rk] = mn;
          }
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_Sfree);
    }
    // ---- combine the lane quarters (a column's keys are spread over all of them)
#pragma unroll
    for (int k = 0; k < NGRP / 2; ++k)
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
        const int i0 = (cs * (NGRP / 2) + k) * QPG;
        const int col = col_of(32 * blk + lane, i0);
        redm[sub * NQT + col] = m_run[2 * k + blk];
        reds[sub * NQT + col] = l_run[2 * k + blk];
      }
    ptx::named_bar_sync(1, 32 * NCW);
    for (int j = ctid; j < NQT; j += 32 * NCW) {
      float m = -INFINITY;
      for (int q = 0; q < 4; ++q) m = fmaxf(m, redm[q * NQT + j]);
      float l = 0.f;
      for (int q = 0; q < 4; ++q) {
        const float mq = redm[q * NQT + j];
        if (mq != -INFINITY) l += reds[q * NQT + j] * exp2f((mq - m) * sl2e);
      }
      mval[j] = m == -INFINITY ? 0.f : m * sl2e;
      linv[j] = l > 0.f ? 1.f / l : 0.f;
    }
    ptx::named_bar_sync(1, 32 * NCW);

    // ---- pass B
    unsigned char *prow = smem + geo.p_off + (key_local & 7) * 16 + (key_local >> 3) * (BM * 16);
    for (int kt = 0; kt < nkt; ++kt) {
      const int s = k_lo + kt * KT_ROWS + key_local;
      const int rows = kt == nkt - 1 ? rlast : KT_ROWS;
      const bool key_ok = s < slen && key_local < rows;
      const bool active = __any_sync(0xffffffffu, key_ok && s <= q0 + BM - 1 &&
                                                      (p.window <= 0 || s >= q0 - p.window + 1));
      if (ok && !ptx::mbar_wait(bar_S, (nkt + kt) & 1, WAIT)) { ok = false; record_err(p, ERR_TIMEOUT_S); }
      if (ok && kt >= 1 && !ptx::mbar_wait(bar_Pfree, (kt - 1) & 1, WAIT)) {
        ok = false;
        record_err(p, ERR_TIMEOUT_P);
      }
      ptx::tc_fence_after();
#pragma unroll 1
      for (int k = 0; k < NGRP / 2; ++k) {
        const int i0 = (cs * (NGRP / 2) + k) * QPG;
        float o0[HPG], o1[HPG];
        if (active && ok) {
          float v0[HPG], v1[HPG];
          compose_pre(i0, s, key_ok, v0, v1);
#pragma unroll
          for (int h = 0; h < HPG; ++h) {
            const int c0 = h * BM + i0;
            v0[h] = v0[h] == -INFINITY ? 0.f : exp2f(fmaf(v0[h], sl2e, -mval[c0])) * linv[c0];
            v1[h] = v1[h] == -INFINITY ? 0.f : exp2f(fmaf(v1[h], sl2e, -mval[c0 + 1])) * linv[c0 + 1];
          }
          compose32x2<E, R>(v0, v1, o0, o1, Wz + HPG * HPG, rec + (BM + i0) * geo.rec_floats,
                            rec + (BM + i0 + 1) * geo.rec_floats, p.post, (int64_t)b * T + s, H, hbase, key_ok);
        } else {
#pragma unroll
          for (int h = 0; h < HPG; ++h) { o0[h] = 0.f; o1[h] = 0.f; }
        }
        if (key_local < rows) {
#pragma unroll
          for (int h = 0; h < HPG; ++h) {
            const E lo = from_f<E>(o0[h]), hi = from_f<E>(o1[h]);
            const uint32_t pk = static_cast<uint32_t>(*reinterpret_cast<const uint16_t *>(&lo)) |
                                (static_cast<uint32_t>(*reinterpret_cast<const uint16_t *>(&hi)) << 16);
            *reinterpret_cast<uint32_t *>(prow + h * (KT_ROWS * BM * 2) + i0 * 2) = pk;
          }
        }
      }
      ptx::fence_proxy_async_smem();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        ptx::mbar_arrive(bar_Sfree);
        ptx::mbar_arrive(bar_P);
      }
    }

    // ---- epilogue: O^T -> SMEM [head][d half][query][64 d] -> TMA store
    if (ok && !ptx::mbar_wait(bar_O, 0, WAIT)) { ok = false; record_err(p, ERR_TIMEOUT_O); }
    ptx::tc_fence_after();
    unsigned char *stage = smem + geo.q_off;
    const int d = key_local;  // same lane <-> row mapping for the two 64-d halves
    if (ok) {
#pragma unroll 1
      for (int h = cs; h < HPG; h += 2) {
        float v[8];
        ptx::tmem_ld<8>(tl + o_col + h * BM, v);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < BM; ++i)
          *reinterpret_cast<E *>(stage + (h * 2 + (d >> 6)) * (BM * 128) + i * 128 + (d & 63) * 2) = from_f<E>(v[i]);
      }
    }
    ptx::fence_proxy_async_smem();
    ptx::named_bar_sync(1, 32 * NCW);
    if (threadIdx.x == 0 && ok) {
      for (int h = 0; h < HPG; ++h)
        for (int c = 0; c < 2; ++c)
          ptx::tma_store_4d(&tm_o, stage + (h * 2 + c) * (BM * 128), c * 64, hbase + h, q0, b);
      ptx::bulk_commit();
      ptx::bulk_wait_read0();
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == tma_warp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tbase, 512);
  }
}

template <typename E, int R>
static cudaError_t launch_t(const dc_attn_params &p, cudaStream_t st) {
  const GeoS32 geo = make_geo_32<R>();
  const size_t smem = geo.total + 1024;
  const int64_t sb = (int64_t)p.T * p.H * D, st_ = (int64_t)p.H * D, sh = D;
  CUtensorMap mq, mk, mv, mo;
  if (!make_map(&mq, p.q, p.dtype, p.B, p.T, p.H, BM, sb, st_, sh, true) ||
      !make_map(&mk, p.k, p.dtype, p.B, p.T, p.H, KT_ROWS, sb, st_, sh, true) ||
      !make_map(&mv, p.v, p.dtype, p.B, p.T, p.H, KT_ROWS, sb, st_, sh, true) ||
      !make_map(&mo, p.out, p.dtype, p.B, p.T, p.H, BM, p.out_sb, p.out_st, p.out_sh, false))
    return cudaErrorInvalidValue;
  TcParams tp;
  tp.B = p.B; tp.T = p.T; tp.H = p.H; tp.G = p.G; tp.window = p.window; tp.slen_default = p.T;
  tp.scale = p.scale;
  tp.seq_lens = p.seq_lens;
  tp.out = p.out;
  tp.out_sb = p.out_sb; tp.out_st = p.out_st; tp.out_sh = p.out_sh;
  tp.err_flag = p.err_flag;
  tp.pre = to_ptrs(p.pre);
  tp.post = to_ptrs(p.post);
  auto kern = dc_tcs32_kernel<E, R>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((p.T + BM - 1) / BM, p.B * p.G);
  kern<<<grid, 32 * (NCW + 2), smem, st>>>(mq, mk, mv, mo, tp);
  return cudaGetLastError();
}

template <typename E>
static cudaError_t launch_e(const dc_attn_params &p, cudaStream_t st) {
  return p.R <= 1 ? launch_t<E, 1>(p, st) : launch_t<E, 2>(p, st);
}

}  // namespace tcs32

bool tcs32_supports(const dc_attn_params &p, std::string *why) {
  auto no = [&](const char *m) { if (why) *why = m; return false; };
  if (p.D != 128) return no("D must be 128");
  if (p.H / p.G != 32) return no("heads per group must be 32");
  if (p.R > 2) return no("rank R > 2");
  if (!(p.scale > 0.f)) return no("non-positive softmax scale");
  if (p.pre.qmat || p.post.qmat) return no("per-query mixing matrices use the SIMT kernel");
  auto al = [](const void *x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  if (!al(p.q) || !al(p.k) || !al(p.v) || !al(p.out)) return no("q, k, v, out must be 16-byte aligned");
  if (p.out_sb % 8 || p.out_st % 8 || p.out_sh % 8) return no("output strides must be multiples of 8 elements");
  // the per-key weights are read 8 heads at a time (16-byte loads)
  if (p.H % 8) return no("H must be a multiple of 8");
  for (const dc_terms *t : {&p.pre, &p.post})
    for (const void *w : {t->kw1, t->kw2, t->kdd})
      if (w && !al(w)) return no("key-wise weights must be 16-byte aligned");
  return true;
}

cudaError_t launch_tcs32(const dc_attn_params &p, cudaStream_t st) {
  if (p.dtype == DC_DTYPE_BF16) return tcs32::launch_e<__nv_bfloat16>(p, st);
  return tcs32::launch_e<__half>(p, st);
}

}  // namespace dcattn
