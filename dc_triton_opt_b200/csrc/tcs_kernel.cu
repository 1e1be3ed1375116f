// Two-pass streaming tensor-core DC-attention forward (sm_100a).
//
// Covers what the single-pass kernels of tc_kernel.cu cannot hold on chip:
// full-causal layers (config 3 of the benchmark) and windows longer than
// three key tiles, at up to 8 heads per group.  One CTA owns (query block, batch, head
// group) and streams the block's key range [k_lo, q0 + BM) in tiles of 128
// keys, twice:
//   pass A  S^T = K Q^T per head (TMEM) -> pre-composition -> mask ->
//           warp-local column max / sum, folded into running per-column
//           statistics (online softmax statistics of the composed logits);
//   combine the running statistics of the four TMEM lane quarters;
//   pass B  S^T again -> pre-composition -> P = exp(S - m) / l ->
//           post-composition -> P' (SMEM) -> O^T += V^T P'^T (TMEM).
// The post-composition mixes normalised probabilities of different heads
// (dc_attention_torch.py:236-248), so every head's statistics must be final
// before any P' exists: hence two passes (the QK products are recomputed on
// the tensor cores, which are far from busy in this op).
// Layout and composition are those of tc_kernel.cu: keys on TMEM lanes,
// (head, query) pairs on columns, one thread per key.
// Warps: 8 compose warps (2 per TMEM lane quarter, splitting the column
// groups), 1 TMA warp, 1 MMA warp; the compose warps also run the epilogue.

#include <cuda.h>
#include <cuda_runtime.h>

#include <string>

#include "tc_common.cuh"

namespace dcattn {
namespace tcs {

using namespace tc;

constexpr int NCW = 8;  // compose warps

template <int HPG>
struct Shape {
  static constexpr int NQT = HPG <= 8 ? 128 : 256;  // (head, query) columns
  static constexpr int BM = NQT / HPG;               // queries per CTA
  static constexpr int GI = 32 / HPG;                // queries per 32-value group
  static constexpr int NG = BM / GI;                 // column groups
  static constexpr int NSB = HPG <= 8 ? 2 : 1;       // S buffers in TMEM
  static constexpr int NPB = HPG <= 8 ? 2 : 1;       // P' buffers in SMEM
  static constexpr int NSLOT = HPG <= 8 ? 3 : 2;     // K/V ring slots
};

struct GeoS {
  int q_off, ring_off, p_off, raw_off, mrec_off, red_off, stat_off, scr_off, bar_off, tmem_off, total;
};

template <int HPG, int R>
__host__ __device__ inline GeoS make_geo_s() {
  using S = Shape<HPG>;
  GeoS g{};
  g.q_off = 0;
  g.ring_off = S::NQT * 256;
  g.p_off = g.ring_off + S::NSLOT * TILE_BYTES;
  int o = g.p_off + S::NPB * KT_ROWS * S::NQT * 2;
  g.raw_off = round_up(o, 16); o = g.raw_off + 2 * S::BM * HPG * (2 * R + 1) * 4;  // per-query weights
  g.mrec_off = round_up(o, 16); o = g.mrec_off + 2 * S::BM * HPG * HPG * 4;        // mixing matrices
  g.red_off = round_up(o, 16); o = g.red_off + 2 * 4 * S::NQT * 4;  // per lane quarter: running max, sum
  g.stat_off = o; o += 2 * S::NQT * 4;                              // combined [query][head]: max, 1 / sum
  g.scr_off = round_up(o, 16); o = g.scr_off + NCW * 64 * 4;        // per warp: 32 maxima, 32 sums
  g.bar_off = round_up(o, 8); o = g.bar_off + 24 * 8;
  g.tmem_off = o; o += 16;
  g.total = o;
  return g;
}

template <typename E, int HPG, int R>
__global__ void __launch_bounds__(32 * (NCW + 2), 1)
    dc_tcs_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                  const TcParams p) {
  using S = Shape<HPG>;
  constexpr int NQT = S::NQT, BM = S::BM, GI = S::GI, NG = S::NG, NSB = S::NSB, NPB = S::NPB,
                NSLOT = S::NSLOT;
  constexpr int GPW = NG / 2;  // column groups per compose warp
  static_assert(NG % 2 == 0, "group split");

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                          ~static_cast<uintptr_t>(1023));
  const GeoS geo = make_geo_s<HPG, R>();
  float *redm = reinterpret_cast<float *>(smem + geo.red_off), *reds = redm + 4 * NQT;
  float *mval = reinterpret_cast<float *>(smem + geo.stat_off), *linv = mval + NQT;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + geo.bar_off);
  uint64_t *bar_full = bars + 0, *bar_free = bars + 3, *bar_q = bars + 6;
  uint64_t *bar_S = bars + 7, *bar_Sfree = bars + 9, *bar_P = bars + 11, *bar_Pfree = bars + 13;
  uint64_t *bar_O = bars + 15;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + geo.tmem_off);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tma_warp = NCW, mma_warp = NCW + 1;
  const int nqb = (p.T + BM - 1) / BM;
  const int qb = nqb - 1 - static_cast<int>(blockIdx.x);  // heaviest (latest) query blocks first
  const int b = blockIdx.y / p.G, g = blockIdx.y % p.G;
  const int q0 = qb * BM, H = p.H, T = p.T, hbase = g * HPG;
  const int k_lo = p.window > 0 ? max(0, q0 - p.window + 1) : 0;
  const int span = min(q0 + BM, T) - k_lo;
  const int nkt = (span + KT_ROWS - 1) / KT_ROWS;
  const int rlast = ((span - KT_ROWS * (nkt - 1)) + 15) / 16 * 16;
  const int slen = p.seq_lens ? min(max(p.seq_lens[b], 0), T) : T;
  const uint32_t WAIT = p.wait_us;
  const uint32_t o_col = NSB * NQT;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 3; ++i) {
      ptx::mbar_init(bar_full + i, 1);
      ptx::mbar_init(bar_free + i, 1);
    }
    ptx::mbar_init(bar_q, 1);
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(bar_S + i, 1);
      ptx::mbar_init(bar_Sfree + i, NCW);
      ptx::mbar_init(bar_P + i, NCW);
      ptx::mbar_init(bar_Pfree + i, 1);
    }
    ptx::mbar_init(bar_O, 1);
    ptx::fence_mbar_init();
  }
  if (warp == tma_warp) ptx::tmem_alloc(tmem_slot, 512);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == tma_warp) {
    // ================================================= TMA producer
    // ring jobs: pass A K(kt, h); pass B K(0, h); then K(kt, h), V(kt-1, h); last V(nkt-1, h)
    if (lane == 0 && !p.skip_loads) {
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
    // ================================================= MMA issuer
    // Whole warp runs the loops; one elected lane issues each tcgen05 op.
    const uint32_t ab_fmt = std::is_same<E, __nv_bfloat16>::value ? 1u : 0u;
    const uint32_t idesc_qk = ptx::idesc_f16(ab_fmt, 0, 0, 128, BM);
    const uint32_t idesc_pv = ptx::idesc_f16(ab_fmt, 1, 1, 128, BM);
    const uint64_t qd0 = ptx::smem_desc(ptx::smem_u32(smem + geo.q_off), 16, 1024, 2);
    const uint64_t kd0 = ptx::smem_desc(ptx::smem_u32(smem + geo.ring_off), 16, 1024, 2);
    const uint64_t vd0 = ptx::smem_desc(ptx::smem_u32(smem + geo.ring_off), TILE_BYTES / 2, 1024, 2);
    const uint64_t pd0 = ptx::smem_desc(ptx::smem_u32(smem + geo.p_off), BM * 16, 128, 0);
    int job = 0;
    bool ok = true;
    auto wait_u = [&](uint64_t *bar, int parity, int code) {
      const bool got = __all_sync(0xffffffffu, ok && ptx::mbar_wait(bar, parity, WAIT));
      if (ok && !got) {
        ok = false;
        if (lane == 0) record_err(p, code);
      }
      return ok;
    };
    wait_u(bar_q, 0, ERR_TIMEOUT_Q);
    ptx::tc_fence_after();
    auto qk = [&](int sidx) {
      const int sb = sidx % NSB;
      if (sidx >= NSB && !wait_u(bar_Sfree + sb, ((sidx - NSB) / NSB) & 1, ERR_TIMEOUT_S)) return;
      ptx::tc_fence_after();
      for (int h = 0; h < HPG && ok; ++h, ++job) {
        const int slot = job % NSLOT;
        if (!wait_u(bar_full + slot, (job / NSLOT) & 1, ERR_TIMEOUT_FULL)) return;
        ptx::tc_fence_after();
        const uint64_t ad = ptx::desc_add(kd0, slot * TILE_BYTES);
        const uint64_t bd = ptx::desc_add(qd0, h * BM * 256);
        const uint32_t dd = tbase + sb * NQT + h * BM;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          if (ptx::elect_one())
            ptx::mma_f16_ss(dd, ptx::desc_add(ad, (ks >> 2) * (TILE_BYTES / 2) + (ks & 3) * 32),
                            ptx::desc_add(bd, (ks >> 2) * (BM * 128) + (ks & 3) * 32), idesc_qk, ks > 0);
        if (ptx::elect_one()) ptx::mma_commit(bar_free + slot);
        __syncwarp();
      }
      if (ptx::elect_one()) ptx::mma_commit(bar_S + sb);
      __syncwarp();
    };
    auto pv = [&](int kt) {
      const int pb = kt % NPB;
      if (!wait_u(bar_P + pb, (kt / NPB) & 1, ERR_TIMEOUT_P)) return;
      ptx::tc_fence_after();
      const int nks = (kt == nkt - 1 ? rlast : KT_ROWS) / 16;
      for (int h = 0; h < HPG && ok; ++h, ++job) {
        const int slot = job % NSLOT;
        if (!wait_u(bar_full + slot, (job / NSLOT) & 1, ERR_TIMEOUT_FULL)) return;
        ptx::tc_fence_after();
        const uint64_t ad = ptx::desc_add(vd0, slot * TILE_BYTES);
        const uint64_t bd = ptx::desc_add(pd0, pb * (KT_ROWS * NQT * 2) + h * (KT_ROWS * BM * 2));
        const uint32_t dd = tbase + o_col + h * BM;
#pragma unroll
        for (int ks = 0; ks < KT_ROWS / 16; ++ks)
          if (ks < nks && ptx::elect_one())
            ptx::mma_f16_ss(dd, ptx::desc_add(ad, ks * 2048), ptx::desc_add(bd, ks * (2 * BM * 16)), idesc_pv,
                            (kt > 0 || ks > 0));
        if (ptx::elect_one()) ptx::mma_commit(bar_free + slot);
        __syncwarp();
      }
      if (ptx::elect_one()) ptx::mma_commit(bar_Pfree + pb);
      __syncwarp();
    };
    for (int kt = 0; kt < nkt && ok; ++kt) qk(kt);
    for (int kt = 0; kt < nkt && ok; ++kt) {
      qk(nkt + kt);
      if (kt >= 1 && ok) pv(kt - 1);
    }
    if (ok) pv(nkt - 1);
    if (ptx::elect_one()) ptx::mma_commit(bar_O);
    __syncwarp();
  } else {
    // ================================================= compose warps
    // Composition as in the single-pass kernels (tc_kernel.cu): per-query
    // mixing matrices M_t built once per CTA (the pre set scaled by
    // scale * log2(e)), key weights in registers, fixed-point warp sums, and
    // two queries per paired-fp32 instruction at 1-4 heads per group.
    constexpr bool PAIR = HPG <= 4;
    constexpr int RAWF = HPG * (2 * R + 1), MF = HPG * HPG, NCK = 2 * R + 1, NCH = 2 * BM * NCK;
    const int sub = warp & 3, cs = warp >> 2;
    const int g_begin = cs * GPW;
    const int s_local = 32 * sub + lane;
    const int ctid = threadIdx.x;  // compose threads are 0 .. 32*NCW-1
    const float sl2e = p.scale * kLog2e;
    float *raw = reinterpret_cast<float *>(smem + geo.raw_off);    // [set][BM][RAWF]
    float *mrec = reinterpret_cast<float *>(smem + geo.mrec_off);  // [set][BM][h'][h] (pair layout with PAIR)
    uint32_t *scr = reinterpret_cast<uint32_t *>(smem + geo.scr_off) + warp * 64;  // this warp's [max | sum] x 32
    auto col_of = [&](int L, int i0) { return (L / GI) * BM + i0 + (L % GI); };
    auto midx = [&](int set, int i, int h1, int h) {
      return PAIR ? set * BM * MF + (i >> 1) * 2 * MF + (h1 * HPG + h) * 2 + (i & 1)
                  : ((set * BM + i) * HPG + h1) * HPG + h;
    };

    for (int c = ctid; c < NCH; c += 32 * NCW) {
      const int set = c / (BM * NCK), rem = c % (BM * NCK), i = rem / NCK, k = rem % NCK;
      const TermPtrs &tm = set ? p.post : p.pre;
      const int t = q0 + i;
      const int64_t tok = (int64_t)b * T + t;
      const E *src = nullptr;
      if (t < T) {
        if (k == 0) src = tm.qdd ? elem<E>(tm.qdd, tok * H + hbase) : nullptr;
        else if (k <= R) src = tm.qw1 ? elem<E>(tm.qw1, (tok * H + hbase) * R + (k - 1) * HPG) : nullptr;
        else src = tm.qw2 ? elem<E>(tm.qw2, (tok * R + (k - 1 - R)) * H + hbase) : nullptr;
      }
      const Raw16<HPG> v = src ? ld_raw16<HPG>(src) : raw16_zero<HPG>();
      float *dst = raw + (set * BM + i) * RAWF + k * HPG;
#pragma unroll
      for (int h = 0; h < HPG; ++h) dst[h] = raw16_get<E, HPG>(v, h);
    }
    ptx::named_bar_sync(1, 32 * NCW);
    for (int idx = ctid; idx < 2 * BM * MF; idx += 32 * NCW) {
      const int set = idx / (BM * MF), i = (idx / MF) % BM, h1 = (idx % MF) / HPG, h = idx % HPG;
      const TermPtrs &tm = set ? p.post : p.pre;
      const float *rr = raw + (set * BM + i) * RAWF;
      float m = (tm.w ? tm.w[((int64_t)g * HPG + h1) * HPG + h] : 0.f) +
                (h1 == h ? (tm.identity ? 1.f : 0.f) + rr[h] : 0.f) + qmat_at<E>(tm, b, q0 + i, T, H, HPG, hbase, h1, h);
#pragma unroll
      for (int r = 0; r < R; ++r) m = fmaf(rr[HPG + h1 * R + r], rr[HPG + HPG * R + r * HPG + h], m);
      mrec[midx(set, i, h1, h)] = set ? m : m * sl2e;
    }
    ptx::named_bar_sync(1, 32 * NCW);

    // per-key weights of the pre (k*) and post (p*) sets; with PAIR also as duplicated pairs
    struct KeyW {
      float w1[HPG * R], w2[R * HPG], dd[HPG];
      ptx::f2_t w1d[HPG * R], w2d[R * HPG], ddd[HPG];
    };
    KeyW kpre, kpost;
    auto load_key = [&](KeyW &kw, const TermPtrs &tm, float f, int64_t tok, bool okk) {
      load_key_weights_vec<E, HPG, R>(tm, tok, H, hbase, okk, kw.w1, kw.w2, kw.dd);
#pragma unroll
      for (int j = 0; j < R * HPG; ++j) kw.w2[j] *= f;
#pragma unroll
      for (int j = 0; j < HPG; ++j) kw.dd[j] *= f;
      if constexpr (PAIR) {
#pragma unroll
        for (int j = 0; j < HPG * R; ++j) kw.w1d[j] = ptx::f2_dup(kw.w1[j]);
#pragma unroll
        for (int j = 0; j < R * HPG; ++j) kw.w2d[j] = ptx::f2_dup(kw.w2[j]);
#pragma unroll
        for (int j = 0; j < HPG; ++j) kw.ddd[j] = ptx::f2_dup(kw.dd[j]);
      }
    };
    // composition of GI queries from i0 (set: pre 0 / post 1) in place on v
    auto compose_group = [&](float (&v)[HPG][GI], int set, int i0, const KeyW &kw) {
      if constexpr (PAIR) {
#pragma unroll
        for (int ii = 0; ii < GI; ii += 2) {
          ptx::f2_t a[HPG], o[HPG];
#pragma unroll
          for (int h = 0; h < HPG; ++h) a[h] = ptx::f2_pack(v[h][ii], v[h][ii + 1]);
          compose_m2<HPG, R>(a, o, mrec + set * BM * MF + (i0 + ii) * MF, kw.w1d, kw.w2d, kw.ddd);
#pragma unroll
          for (int h = 0; h < HPG; ++h) {
            v[h][ii] = ptx::f2_lo(o[h]);
            v[h][ii + 1] = ptx::f2_hi(o[h]);
          }
        }
      } else {
#pragma unroll
        for (int ii = 0; ii < GI; ++ii) {
          float a[HPG], o[HPG];
#pragma unroll
          for (int h = 0; h < HPG; ++h) a[h] = v[h][ii];
          compose_m<HPG, R>(a, o, mrec + set * BM * MF + (i0 + ii) * MF, kw.w1, kw.w2, kw.dd);
#pragma unroll
          for (int h = 0; h < HPG; ++h) v[h][ii] = o[h];
        }
      }
    };
    float m_run[GPW], l_run[GPW];  // running statistics of column `lane` of each group
#pragma unroll
    for (int k = 0; k < GPW; ++k) { m_run[k] = kMaskedLogit; l_run[k] = 0.f; }
    bool ok = true;

    // ---- pass A: running column statistics of the composed logits
    for (int kt = 0; kt < nkt; ++kt) {
      const int sidx = kt, sb = sidx % NSB;
      const int s = k_lo + kt * KT_ROWS + s_local;
      const int rows = kt == nkt - 1 ? rlast : KT_ROWS;
      const bool key_ok = s < slen && s_local < rows;
      const int wk0 = k_lo + kt * KT_ROWS + 32 * sub;
      const bool active = 32 * sub < rows && wk0 <= min(q0 + BM - 1, slen - 1) &&
                          (p.window <= 0 || wk0 + 31 >= q0 - p.window + 1);
      const bool keys_in = wk0 + 31 < slen && 32 * sub + 31 < rows;
      auto all_valid = [&](int t0) {
        return keys_in && wk0 + 31 <= t0 && (p.window <= 0 || t0 + GI - 1 - wk0 < p.window) && t0 + GI - 1 < T;
      };
      auto valid = [&](int t) { return key_ok && s <= t && (p.window <= 0 || t - s < p.window) && t < T; };
      if (active) load_key(kpre, p.pre, sl2e, (int64_t)b * T + s, key_ok);
      if (ok && !ptx::mbar_wait(bar_S + sb, (sidx / NSB) & 1, WAIT)) { ok = false; record_err(p, ERR_TIMEOUT_S); }
      ptx::tc_fence_after();
      const uint32_t tl = tbase + (static_cast<uint32_t>(32 * sub) << 16) + sb * NQT;
#pragma unroll 1
      for (int k = 0; k < GPW; ++k) {
        const int i0 = (g_begin + k) * GI;
        if (!(active && ok)) {
          // nothing of this warp survives the mask: no change to the statistics
          continue;
        }
        float v[HPG][GI];
#pragma unroll
        for (int h = 0; h < HPG; ++h) ptx::tmem_ld<GI>(tl + h * BM + i0, v[h]);
        ptx::tmem_wait_ld();
        compose_group(v, 0, i0, kpre);
        if (!all_valid(q0 + i0)) {
#pragma unroll
          for (int ii = 0; ii < GI; ++ii) {
            const bool vl = valid(q0 + i0 + ii);
#pragma unroll
            for (int h = 0; h < HPG; ++h) v[h][ii] = vl ? v[h][ii] : kMaskedLogit;
          }
        }
        // warp-local max and fixed-point sum of each column (value L = h * GI + ii)
#pragma unroll
        for (int h = 0; h < HPG; ++h)
#pragma unroll
          for (int ii = 0; ii < GI; ++ii) {
            const float mw = ptx::warp_max(v[h][ii]);
            const uint32_t sw = ptx::warp_sum_u32(__float_as_uint(ptx::ex2(v[h][ii] - mw) + 1.f));
            if (lane == 0) {
              scr[h * GI + ii] = __float_as_uint(mw);
              scr[32 + h * GI + ii] = sw;
            }
          }
        __syncwarp();
        // lane L folds column L's (max, sum) of this tile into its running statistics
        const float mt = __uint_as_float(scr[lane]);
        const float st = static_cast<float>(scr[32 + lane] - 32u * 0x3F800000u) * 0x1p-23f;
        __syncwarp();
        const float mn = fmaxf(m_run[k], mt);
        l_run[k] = l_run[k] * ptx::ex2(m_run[k] - mn) + st * ptx::ex2(mt - mn);
        m_run[k] = mn;
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_Sfree + sb);
    }
    // ---- combine the four lane quarters of every column; statistics in [query][head]
#pragma unroll
    for (int k = 0; k < GPW; ++k) {
      const int col = col_of(lane, (g_begin + k) * GI);
      redm[sub * NQT + col] = m_run[k];
      reds[sub * NQT + col] = l_run[k];
    }
    ptx::named_bar_sync(1, 32 * NCW);
    for (int j = ctid; j < NQT; j += 32 * NCW) {
      float m = kMaskedLogit;
      for (int q = 0; q < 4; ++q) m = fmaxf(m, redm[q * NQT + j]);
      float l = 0.f;
      for (int q = 0; q < 4; ++q) l += reds[q * NQT + j] * ptx::ex2(redm[q * NQT + j] - m);
      const int h = j / BM, i = j % BM;
      const bool dead = !(m > 0.5f * kMaskedLogit && l > 0.f);  // every key masked: output 0
      mval[i * HPG + h] = dead ? 0.f : m;
      linv[i * HPG + h] = dead ? 0.f : __frcp_rn(l);
    }
    ptx::named_bar_sync(1, 32 * NCW);

    // ---- pass B: normalised probabilities, post-composition, P' -> SMEM
    for (int kt = 0; kt < nkt; ++kt) {
      const int sidx = nkt + kt, sb = sidx % NSB, pb = kt % NPB;
      const int s = k_lo + kt * KT_ROWS + s_local;
      const int rows = kt == nkt - 1 ? rlast : KT_ROWS;
      const bool key_ok = s < slen && s_local < rows;
      const int wk0 = k_lo + kt * KT_ROWS + 32 * sub;
      const bool active = 32 * sub < rows && wk0 <= min(q0 + BM - 1, slen - 1) &&
                          (p.window <= 0 || wk0 + 31 >= q0 - p.window + 1);
      const bool keys_in = wk0 + 31 < slen && 32 * sub + 31 < rows;
      auto all_valid = [&](int t0) {
        return keys_in && wk0 + 31 <= t0 && (p.window <= 0 || t0 + GI - 1 - wk0 < p.window) && t0 + GI - 1 < T;
      };
      auto valid = [&](int t) { return key_ok && s <= t && (p.window <= 0 || t - s < p.window) && t < T; };
      if (active) {
        load_key(kpre, p.pre, sl2e, (int64_t)b * T + s, key_ok);
        load_key(kpost, p.post, 1.f, (int64_t)b * T + s, key_ok);
      }
      if (ok && !ptx::mbar_wait(bar_S + sb, (sidx / NSB) & 1, WAIT)) { ok = false; record_err(p, ERR_TIMEOUT_S); }
      // P' buffer pb was last read by the PV of tile kt - NPB
      if (ok && kt >= NPB && !ptx::mbar_wait(bar_Pfree + pb, ((kt - NPB) / NPB) & 1, WAIT)) {
        ok = false;
        record_err(p, ERR_TIMEOUT_P);
      }
      ptx::tc_fence_after();
      const uint32_t tl = tbase + (static_cast<uint32_t>(32 * sub) << 16) + sb * NQT;
      unsigned char *prow = smem + geo.p_off + pb * (KT_ROWS * NQT * 2) + (s_local & 7) * 16 + (s_local >> 3) * (BM * 16);
#pragma unroll 1
      for (int k = 0; k < GPW; ++k) {
        const int i0 = (g_begin + k) * GI;
        float v[HPG][GI];
        if (active && ok) {
#pragma unroll
          for (int h = 0; h < HPG; ++h) ptx::tmem_ld<GI>(tl + h * BM + i0, v[h]);
          ptx::tmem_wait_ld();
          compose_group(v, 0, i0, kpre);
          const bool full = all_valid(q0 + i0);
#pragma unroll
          for (int ii = 0; ii < GI; ++ii) {
            float mv[HPG], li[HPG];
            ld_row<HPG>(mval + (i0 + ii) * HPG, mv);
            ld_row<HPG>(linv + (i0 + ii) * HPG, li);
            const bool vl = full || valid(q0 + i0 + ii);
#pragma unroll
            for (int h = 0; h < HPG; ++h) v[h][ii] = vl ? ptx::ex2(v[h][ii] - mv[h]) * li[h] : 0.f;
          }
          compose_group(v, 1, i0, kpost);
        } else {
#pragma unroll
          for (int h = 0; h < HPG; ++h)
#pragma unroll
            for (int ii = 0; ii < GI; ++ii) v[h][ii] = 0.f;
        }
        if (s_local < rows) {
#pragma unroll
          for (int h = 0; h < HPG; ++h) {
            unsigned char *tile = prow + h * (KT_ROWS * BM * 2);
#pragma unroll
            for (int c = 0; c < GI; c += 8 < GI ? 8 : GI) {
              constexpr int W8 = GI < 8 ? GI : 8;
              uint32_t pk[W8 / 2];
#pragma unroll
              for (int u = 0; u < W8 / 2; ++u) pk[u] = pack2<E>(v[h][c + 2 * u], v[h][c + 2 * u + 1]);
              const int i = i0 + c;
              unsigned char *dst = tile + (i >> 3) * 128 + (i & 7) * 2;
              if constexpr (W8 == 8) {
                *reinterpret_cast<uint4 *>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
              } else if constexpr (W8 == 4) {
                *reinterpret_cast<uint2 *>(dst) = make_uint2(pk[0], pk[1]);
              } else {
                *reinterpret_cast<uint32_t *>(dst) = pk[0];
              }
            }
          }
        }
      }
      ptx::fence_proxy_async_smem();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        ptx::mbar_arrive(bar_Sfree + sb);
        ptx::mbar_arrive(bar_P + pb);
      }
    }

    // ---- epilogue: O^T (lanes = d) -> SMEM [head][d half][query][64 d] -> TMA store
    if (ok && !ptx::mbar_wait(bar_O, 0, WAIT)) { ok = false; record_err(p, ERR_TIMEOUT_O); }
    ptx::tc_fence_after();
    unsigned char *stage = smem + geo.q_off;  // Q is dead once every MMA has completed
    const int d = 32 * sub + lane;
    if (ok) {
#pragma unroll 1
      for (int c = cs; c < NQT / 8; c += 2) {
        float v[8];
        ptx::tmem_ld<8>(tbase + (static_cast<uint32_t>(32 * sub) << 16) + o_col + 8 * c, v);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const int col = 8 * c + jj, h = col / BM, i = col % BM;
          *reinterpret_cast<E *>(stage + (h * 2 + (d >> 6)) * (BM * 128) + i * 128 + (d & 63) * 2) =
              from_f<E>(v[jj]);
        }
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

template <typename E, int HPG, int R>
static cudaError_t launch_t(const dc_attn_params &p, cudaStream_t st) {
  using S = Shape<HPG>;
  const GeoS geo = make_geo_s<HPG, R>();
  const size_t smem = geo.total + 1024;
  const int64_t sb = (int64_t)p.T * p.H * D, st_ = (int64_t)p.H * D, sh = D;
  CUtensorMap mq, mk, mv, mo;
  if (!make_map(&mq, p.q, p.dtype, p.B, p.T, p.H, S::BM, sb, st_, sh, true) ||
      !make_map(&mk, p.k, p.dtype, p.B, p.T, p.H, KT_ROWS, sb, st_, sh, true) ||
      !make_map(&mv, p.v, p.dtype, p.B, p.T, p.H, KT_ROWS, sb, st_, sh, true) ||
      !make_map(&mo, p.out, p.dtype, p.B, p.T, p.H, S::BM, p.out_sb, p.out_st, p.out_sh, false))
    return cudaErrorInvalidValue;
  TcParams tp;
  tp.B = p.B; tp.T = p.T; tp.H = p.H; tp.G = p.G; tp.window = p.window; tp.slen_default = p.T;
  tp.scale = p.scale;
  tp.seq_lens = p.seq_lens;
  tp.out = p.out;
  tp.out_sb = p.out_sb; tp.out_st = p.out_st; tp.out_sh = p.out_sh;
  tp.err_flag = p.err_flag;
  tp.wait_us = p.wait_us;
  tp.skip_loads = (p.test_flags & DC_TEST_SKIP_LOADS) != 0;
  tp.pre = to_ptrs(p.pre);
  tp.post = to_ptrs(p.post);
  auto kern = dc_tcs_kernel<E, HPG, R>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((p.T + S::BM - 1) / S::BM, p.B * p.G);
  kern<<<grid, 32 * (NCW + 2), smem, st>>>(mq, mk, mv, mo, tp);
  return cudaGetLastError();
}

template <typename E, int HPG>
static cudaError_t launch_r(const dc_attn_params &p, cudaStream_t st) {
  return p.R <= 1 ? launch_t<E, HPG, 1>(p, st) : launch_t<E, HPG, 2>(p, st);
}

template <typename E>
static cudaError_t launch_e(const dc_attn_params &p, cudaStream_t st) {
  switch (p.H / p.G) {
    case 1: return launch_r<E, 1>(p, st);
    case 2: return launch_r<E, 2>(p, st);
    case 4: return launch_r<E, 4>(p, st);
    case 8: return launch_r<E, 8>(p, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace tcs

bool tcs_supports(const dc_attn_params &p, std::string *why) {
  auto no = [&](const char *m) { if (why) *why = m; return false; };
  const int HPG = p.H / p.G;
  if (p.D != 128) return no("D must be 128");
  // (16 heads per group: the per-query mixing matrices do not fit beside the
  // rings; those layers run on the kernel with the static mix on tensor cores)
  if (HPG != 1 && HPG != 2 && HPG != 4 && HPG != 8) return no("heads per group must be 1, 2, 4 or 8");
  if (p.R > 2) return no("rank R > 2");
  if (!(p.scale > 0.f)) return no("non-positive softmax scale");
  auto al = [](const void *x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  if (!al(p.q) || !al(p.k) || !al(p.v) || !al(p.out)) return no("q, k, v, out must be 16-byte aligned");
  if (p.out_sb % 8 || p.out_st % 8 || p.out_sh % 8) return no("output strides must be multiples of 8 elements");
  return true;
}

cudaError_t launch_tcs(const dc_attn_params &p, cudaStream_t st) {
  if (p.dtype == DC_DTYPE_BF16) return tcs::launch_e<__nv_bfloat16>(p, st);
  return tcs::launch_e<__half>(p, st);
}

}  // namespace dcattn
