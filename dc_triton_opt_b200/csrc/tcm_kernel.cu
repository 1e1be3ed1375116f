// Two-pass streaming DC-attention forward with the static head mix on the
// tensor cores, for 16 or 32 heads per group (sm_100a).
//
// At 16-32 heads per group the static HPG x HPG mix costs HPG^2 MACs per
// (query, key) pair, as much as QK^T itself; on CUDA cores it dominates the
// kernel.  Here it is a tcgen05 MMA per query:
//     D_i[key, h] = sum_h' A_i[key, h'] W[h', h]     (M = 64 keys, K = HPG)
// where A_i is the (pre-composition logits | probabilities) tile of query i,
// written by the compose threads to shared memory as fp16.  The diagonal of W,
// the query- and key-wise rank-R terms and the qdd/kdd gates stay on the CUDA
// cores in fp32; only the off-diagonal mix (|W| ~ 0.02) is rounded to fp16.
//
// Tiles and TMEM (512 columns x 128 lanes), BM = 256 / HPG queries per CTA:
//   S  [0,128)    QK^T of a 64-key tile: head h is an M = 64 MMA whose rows
//                 land in lane half h / (HPG/2) of every lane quarter, column
//                 (h % (HPG/2)) * BM + query.  Thread (quarter q, lane l) thus
//                 holds key 16 q + l % 16 for the heads of half l / 16.
//   D  [128,256)  mix output: query i, output half v at lane half v, columns
//                 128 + i * HPG/2 + (h % (HPG/2)); same thread <-> key mapping.
//   O  [256,512)  O^T: head h, d half c (lane half c), column 256 + h*BM + i.
// Pass A: QK, pre mix, running softmax statistics per (head, query).
// Pass B: QK, pre mix, normalise, post mix, P' -> PV.
// Math follows dc_attention_torch.py:159-258 (grouped residual form) extended
// to the static-W / rank-R / gate terms of the general DC formulation.

#include <cuda.h>
#include <cuda_runtime.h>

#include <string>
#include <type_traits>

#include "tc_common.cuh"

namespace dcattn {
namespace tcm {

using namespace tc;

constexpr int KT = 64;             // keys per tile
constexpr int KJOB = KT * 256;     // one ring job: one head, 64 keys x 128 d
constexpr int NCW = 8;             // compose warps (2 per lane quarter)
// K/V staging.  The K, V and P' buffers share one shared-memory pool; a K job
// carries one head's 64-key K tile plus that head's Q rows (the QK^T B
// operand), so no Q copy stays resident.  Separate K and V rings, each with
// one producer lane and one MMA warp consuming it in order (an mbarrier parity
// wait is only unambiguous for a consumer at most one phase behind, so a ring
// never has two consumers).  Pass A streams K alone, so its ring spans the
// whole pool; pass B has NSK K slots, NSV V slots and P'.  With per-query
// mixing matrices (the decomposed form, QM) every query has its own mix B
// operands, and the pass-B K ring gives up two slots for them.
constexpr int NSK_MAX = 5, NSV = 3;
constexpr int NLV = 3;  // issuing lanes of the V producer (<= slots)
__host__ __device__ constexpr int nsk_of(bool qm) { return qm ? 3 : 5; }
__host__ __device__ constexpr int nlk_of(bool qm) { return qm ? 3 : 4; }  // K producer lanes (<= slots)
static_assert(nlk_of(false) <= nsk_of(false) && nlk_of(true) <= nsk_of(true) && NLV <= NSV,
              "a producer round may not wrap its ring");
// Heads whose MMAs are interleaved: the K steps of one head accumulate into one
// TMEM tile and serialise, so independent heads are issued K step by K step.
constexpr int HJ = 1;
static_assert(nsk_of(true) >= HJ && NSV >= HJ, "an interleaved group needs its jobs resident");
constexpr int NKA_MAX = 10;
constexpr uint32_t S_COL = 0, D_COL = 128, O_COL = 256;
// Pass A double-buffers S in the O columns (idle until pass B): S tile n of
// pass A uses buffer n & 1; pass B uses buffer 0 only.
__host__ __device__ constexpr uint32_t s_col(int buf) { return buf ? O_COL : S_COL; }

template <int HPG, bool QM = false>
struct Shape {
  static constexpr int NSK = nsk_of(QM), NLK = nlk_of(QM);
  static constexpr int BM = 256 / HPG;        // queries per CTA
  static constexpr int HH = HPG / 2;          // heads per lane half
  static constexpr int NQG = 64 / HPG;        // queries per compose sub-group (32 values per thread)
  static constexpr int NSG = (BM / 2) / NQG;  // sub-groups per compose warp
  static constexpr int KB = HPG / 8;          // 16-byte k-blocks per mix-operand row
  static constexpr int ATILE = KT * HPG * 2;  // bytes of one query's mix operand
  static constexpr int PHEAD = KT * BM * 2;   // bytes of one head's P' tile
  static constexpr int NCOL = HPG * BM;       // (head, query) columns
  static constexpr int KQJOB = KJOB + BM * 256;              // K tile + Q rows of one head
  static constexpr int VOFF = NSK * KQJOB;                   // V ring in the pool
  static constexpr int POFF = VOFF + NSV * KJOB;             // P' in the pool
  static constexpr int POOL = POFF + HPG * PHEAD;
  static constexpr int NKA = POOL / KQJOB;                   // pass-A K slots
  static_assert(KQJOB % 1024 == 0 && VOFF % 1024 == 0 && POFF % 1024 == 0, "128B-swizzle atoms");
  static_assert(NKA <= NKA_MAX, "barrier space");
};

struct GeoM {
  int p_off, a_off, bm_off, rec_off, stat_off, bar_off, tmem_off, total, recf;
};

template <int HPG, int R, bool QM>
__host__ __device__ inline GeoM make_geo_m() {
  using SH = Shape<HPG, QM>;
  GeoM g{};
  g.p_off = SH::POFF;                           // P': HPG x 64 keys x BM (32 KB); pass-A stats exchange
  g.a_off = SH::POOL;                           // mix operands, BM x 64 keys x HPG fp16 (32 KB)
  g.bm_off = g.a_off + SH::BM * SH::ATILE;      // mix B operands: 2 sets x [BM queries with QM] x HPG x HPG fp16
  int o = g.bm_off + 2 * (QM ? SH::BM : 1) * HPG * HPG * 2;
  g.recf = round_up(HPG * (2 * R + 1), 4);
  g.rec_off = round_up(o, 16); o = g.rec_off + 2 * SH::BM * g.recf * 4;
  g.stat_off = o; o += 2 * SH::NCOL * 4;
  g.bar_off = round_up(o, 8); o = g.bar_off + (2 * (NKA_MAX + NSK_MAX + NSV) + 16) * 8;
  g.tmem_off = o; o += 16;
  g.total = o;
  return g;
}

// The key-wise weights of one key for the HH heads of a lane half, packed as
// loaded (bf16/fp16); issued at the start of a tile, unpacked where used.
template <int HH, int R>
struct KeyW {
  uint4 w1[HH * R / 8];  // kw1[tok, h, r]   flat (h, r)
  uint4 w2[R * HH / 8];  // kw2[tok, r, h]   flat (r, h)
  uint4 dd[HH / 8];      // kdd[tok, h]
};

template <typename E>
__device__ __forceinline__ float unpack_e(const uint4 *v, int j) {
  const E *e = reinterpret_cast<const E *>(v + j / 8);
  return to_f<E>(e[j % 8]);
}

template <typename E, int HH, int R>
__device__ __forceinline__ void load_keyw(KeyW<HH, R> &kw, const TermPtrs &tm, int64_t tok, int H, int h0,
                                          bool key_ok) {
  const uint4 z = make_uint4(0, 0, 0, 0);
  const bool k1 = key_ok && tm.kw1, kd = key_ok && tm.kdd;
  const uint4 *w1 = reinterpret_cast<const uint4 *>(reinterpret_cast<const E *>(tm.kw1) + (tok * H + h0) * R);
  const uint4 *dd = reinterpret_cast<const uint4 *>(reinterpret_cast<const E *>(tm.kdd) + tok * H + h0);
#pragma unroll
  for (int c = 0; c < HH * R / 8; ++c) kw.w1[c] = k1 ? __ldg(w1 + c) : z;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const uint4 *w2 = reinterpret_cast<const uint4 *>(reinterpret_cast<const E *>(tm.kw2) + (tok * R + r) * H + h0);
#pragma unroll
    for (int c = 0; c < HH / 8; ++c) kw.w2[r * (HH / 8) + c] = k1 ? __ldg(w2 + c) : z;
  }
#pragma unroll
  for (int c = 0; c < HH / 8; ++c) kw.dd[c] = kd ? __ldg(dd + c) : z;
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}

template <typename E>
__device__ __forceinline__ uint32_t pack_e2(float lo, float hi) {
  const E a = from_f<E>(lo), b = from_f<E>(hi);
  return static_cast<uint32_t>(*reinterpret_cast<const uint16_t *>(&a)) |
         (static_cast<uint32_t>(*reinterpret_cast<const uint16_t *>(&b)) << 16);
}

template <typename E, int HPG, int R, bool QM>
__global__ void __launch_bounds__(32 * (NCW + 4), 1)
    dc_tcm_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                  const TcParams p) {
  using SH = Shape<HPG, QM>;
  constexpr int NSK = SH::NSK, NLK = SH::NLK;
  constexpr int BM = SH::BM, HH = SH::HH, NQG = SH::NQG, NSG = SH::NSG, KB = SH::KB;
  constexpr int ATILE = SH::ATILE, PHEAD = SH::PHEAD, NCOL = SH::NCOL;
  static_assert(HH * NQG == 32, "a compose sub-group is 32 values per thread");

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                          ~static_cast<uintptr_t>(1023));
  const GeoM geo = make_geo_m<HPG, R, QM>();
  const int recf = geo.recf;
  float *rec = reinterpret_cast<float *>(smem + geo.rec_off);
  float *redm = reinterpret_cast<float *>(smem + geo.p_off), *reds = redm + 4 * NCOL;
  float *mval = reinterpret_cast<float *>(smem + geo.stat_off), *linv = mval + NCOL;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + geo.bar_off);
  constexpr int NKA = SH::NKA, KQJOB = SH::KQJOB;
  uint64_t *bar_afull = bars + 0, *bar_afree = bar_afull + NKA;        // pass-A K ring
  uint64_t *bar_kfull = bar_afree + NKA, *bar_kfree = bar_kfull + NSK;  // pass-B K ring
  // bar_vgo: the pass-A ring is drained, the V ring may start (one phase)
  uint64_t *bar_vfull = bar_kfree + NSK, *bar_vfree = bar_vfull + NSV, *bar_vgo = bar_vfree + NSV;
  uint64_t *bar_q = bar_vgo;  // base of the remaining barriers
  uint64_t *bar_S = bar_q + 1, *bar_Sfree = bar_q + 3;  // two S buffers each
  uint64_t *bar_P = bar_q + 5, *bar_Pfree = bar_q + 6, *bar_O = bar_q + 7;
  uint64_t *bar_A = bar_q + 8, *bar_D = bar_q + 12;  // per compose sub-group (4 each)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + geo.tmem_off);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tma_warp = NCW, mma_warp = NCW + 1, pv_warp = NCW + 2, mix_warp = NCW + 3;
  // Heads are visited in a per-CTA rotated order, so CTAs that run together
  // (neighbouring query blocks, overlapping key spans) read different heads'
  // K/V rows at any moment instead of hitting the same lines.
  const int hrot = (blockIdx.x * 7) % HPG;
  // byte offset of K slot `slot` of the pass-A (ring_a) or pass-B ring
  // (both K rings start at the pool base with the same slot size)
  auto kslot_off = [&](bool, int slot) { return slot * KQJOB; };
  const int nqb = (p.T + BM - 1) / BM;
  const int qb = nqb - 1 - static_cast<int>(blockIdx.x);  // longest spans first
  const int b = blockIdx.y / p.G, g = blockIdx.y % p.G;
  const int q0 = qb * BM, H = p.H, T = p.T, hbase = g * HPG;
  const int k_lo = p.window > 0 ? max(0, q0 - p.window + 1) : 0;
  const int span = min(q0 + BM, T) - k_lo;
  const int nkt = (span + KT - 1) / KT;
  const int rlast = ((span - KT * (nkt - 1)) + 15) / 16 * 16;
  const int slen = p.seq_lens ? min(max(p.seq_lens[b], 0), T) : T;
  const uint32_t WAIT = p.wait_us;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NKA; ++i) {
      ptx::mbar_init(bar_afull + i, 1);
      ptx::mbar_init(bar_afree + i, 1);
    }
    for (int i = 0; i < NSK; ++i) {
      ptx::mbar_init(bar_kfull + i, 1);
      ptx::mbar_init(bar_kfree + i, 1);
    }
    for (int i = 0; i < NSV; ++i) {
      ptx::mbar_init(bar_vfull + i, 1);
      ptx::mbar_init(bar_vfree + i, 1);
    }
    ptx::mbar_init(bar_vgo, 1);
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(bar_S + i, 1);
      ptx::mbar_init(bar_Sfree + i, NCW);
    }
    ptx::mbar_init(bar_P, NCW);
    ptx::mbar_init(bar_Pfree, 1);
    ptx::mbar_init(bar_O, 1);
    for (int i = 0; i < 4; ++i) {
      ptx::mbar_init(bar_A + i, 4);
      ptx::mbar_init(bar_D + i, 1);
    }
    ptx::fence_mbar_init();
  }
  if (warp == tma_warp) ptx::tmem_alloc(tmem_slot, 512);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == tma_warp) {
    // ============================================================ TMA producers
    // Lanes 0-3 fill the K ring (pass A K(0..nkt-1), then pass B K(0..nkt-1)),
    // lanes 16-18 the V ring (V(0..nkt-1)).  A job is one head: a single 5-D
    // box for K (both d halves) plus one for that head's Q rows, or one box
    // for V.  A thread's TMA operations are processed one after another, so
    // consecutive jobs go to different lanes; the lanes of a group advance
    // together, one job each per round, and a group never has more lanes
    // than its ring has slots, so the job a slot waits for was issued in an
    // earlier round.
    const bool isv = lane >= 16;
    const int gl = lane & 15;
    const int L = isv ? NLV : NLK;
    const uint32_t gmask = isv ? (((1u << NLV) - 1) << 16) : ((1u << NLK) - 1);
    if (gl < L && !p.skip_loads) {
      if (gl == 0) {
        if (!isv) {
          ptx::tma_prefetch_desc(&tm_q);
          ptx::tma_prefetch_desc(&tm_k);
        } else {
          ptx::tma_prefetch_desc(&tm_v);
        }
      }
      bool ok = true;
      // jobs [0, njobs) of one ring; job i = head i % HPG of key tile i / HPG
      auto run_ring = [&](int njobs, uint64_t *full, uint64_t *freeb, int nslot, bool ring_a) {
        for (int j0 = 0; j0 < njobs; j0 += L) {
          const int job = j0 + gl;
          bool good = ok;
          if (job < njobs && good) {
            const int kt = job / HPG, h = (job % HPG + hrot) % HPG;
            const int slot = job % nslot, use = job / nslot;
            if (use > 0 && !ptx::mbar_wait(freeb + slot, (use - 1) & 1, WAIT)) good = false;
            if (good) {
              ptx::mbar_expect_tx(full + slot, KJOB + (isv ? 0 : BM * 256));
              unsigned char *dst = smem + (isv ? SH::VOFF + slot * KJOB : kslot_off(ring_a, slot));
              ptx::tma_load_5d(dst, isv ? &tm_v : &tm_k, full + slot, 0, k_lo + kt * KT, 0, hbase + h, b);
              if (!isv) ptx::tma_load_5d(dst + KJOB, &tm_q, full + slot, 0, q0, 0, hbase + h, b);
            }
          }
          const bool all = __all_sync(gmask, good);
          if (ok && !all) {
            ok = false;
            if (gl == 0) record_err(p, ERR_TIMEOUT_FREE);
          }
        }
      };
      if (isv) {
        // the V ring overlaps pass-A slots: start once the K group has seen
        // them drained (a one-phase barrier, so the wait is unambiguous)
        const bool got = __all_sync(gmask, ptx::mbar_wait(bar_vgo, 0, WAIT));
        if (!got) {
          ok = false;
          if (gl == 0) record_err(p, ERR_TIMEOUT_FREE);
        }
        if (ok) run_ring(nkt * HPG, bar_vfull, bar_vfree, NSV, false);
      } else {
        const int na = nkt * HPG;
        run_ring(na, bar_afull, bar_afree, NKA, true);
        // The pass-B K slots and the V ring overlap pass-A slots: wait for the
        // last use of every pass-A slot.  Every job of the ring has been issued
        // (rounds are lockstep) and each issue waited for the slot's previous
        // release, so the last phase cannot be more than one ahead: its
        // parity is unambiguous.
        for (int sl = gl; sl < NKA && ok; sl += L)
          if (sl < na) {
            const int j = sl + ((na - 1 - sl) / NKA) * NKA;
            if (!ptx::mbar_wait(bar_afree + sl, (j / NKA) & 1, WAIT)) ok = false;
          }
        const bool all = __all_sync(gmask, ok);
        if (!all) {
          ok = false;
          if (gl == 0) record_err(p, ERR_TIMEOUT_FREE);
        }
        if (gl == 0) ptx::mbar_arrive(bar_vgo);
        if (ok) run_ring(na, bar_kfull, bar_kfree, NSK, false);
      }
    }
    __syncwarp();
  } else if (warp == mma_warp || warp == pv_warp || warp == mix_warp) {
    // ============================================================ MMA issuers
    // Three warps: QK^T, P'V and the head mixes, so no chain waits behind
    // another (the mixes sit on the compose threads' critical path).  Each warp runs its loops converged and one
    // elected lane issues each tcgen05 instruction; descriptors are bases plus
    // compile-time offsets.  Ring jobs (K or V of one head) are consumed by
    // index, in the producer's order.
    const uint32_t ab_fmt = std::is_same<E, __nv_bfloat16>::value ? 1u : 0u;
    const uint32_t idesc_qk = ptx::idesc_f16(ab_fmt, 0, 0, 64, BM);
    const uint32_t idesc_pv = ptx::idesc_f16(ab_fmt, 1, 1, 64, BM);
    const uint32_t idesc_mix = ptx::idesc_f16(0, 0, 0, 64, HH);  // fp16 x fp16
    const uint64_t dsm = ptx::smem_desc(ptx::smem_u32(smem), 16, 1024, 2);  // K: K-major SW128, + slot offset
    const uint64_t dv0 = ptx::smem_desc(ptx::smem_u32(smem + SH::VOFF), KJOB / 2, 1024, 2);  // V: MN-major
    const uint64_t dp0 = ptx::smem_desc(ptx::smem_u32(smem + geo.p_off), BM * 16, 128, 0);  // P': MN-major
    const uint64_t da0 = ptx::smem_desc(ptx::smem_u32(smem + geo.a_off), 128, KB * 128, 0); // mix A: K-major
    const uint64_t db0 = ptx::smem_desc(ptx::smem_u32(smem + geo.bm_off), 128, KB * 128, 0);
    bool ok = true;
    auto wait_u = [&](uint64_t *bar, int parity, int code) {
      const bool got = __all_sync(0xffffffffu, ok && ptx::mbar_wait(bar, parity, WAIT));
      if (ok && !got) {
        ok = false;
        if (lane == 0) record_err(p, code);
      }
    };
    // ring jobs are consumed in order: wait for a job's data, release its slot
    auto wait_jobs = [&](int job, uint64_t *full, int nslot) {
      for (int hh = 0; hh < HJ; ++hh)
        wait_u(full + ((job + hh) % nslot), ((job + hh) / nslot) & 1, ERR_TIMEOUT_FULL);
      ptx::tc_fence_after();
    };
    auto free_jobs = [&](int job, uint64_t *freeb, int nslot) {
      if (ptx::elect_one())
        for (int hh = 0; hh < HJ; ++hh) ptx::mma_commit(freeb + ((job + hh) % nslot));
      __syncwarp();
    };
    // one round of head mixes (set 0 = pre, 1 = post) for the four sub-groups
    auto mixes = [&](int set, int round) {
      for (int sgl = 0; sgl < NSG; ++sgl)
        for (int cs = 0; cs < 2; ++cs) {
          const int sg = cs * NSG + sgl;
          wait_u(bar_A + sg, round & 1, ERR_TIMEOUT_P);
          if (!ok) return;
          ptx::tc_fence_after();
          const uint64_t aq = ptx::desc_add(da0, sg * NQG * ATILE);
          const uint64_t bq = ptx::desc_add(db0, (QM ? set * BM + sg * NQG : set) * (HPG * HPG * 2));
          const uint32_t dq = tbase + D_COL + sg * NQG * HH;
#pragma unroll
          for (int ks = 0; ks < HPG / 16; ++ks)
#pragma unroll
            for (int ii = 0; ii < NQG; ++ii)
#pragma unroll
              for (int v = 0; v < 2; ++v)
                if (ptx::elect_one())
                  ptx::mma_f16_ss(dq + (static_cast<uint32_t>(16 * v) << 16) + ii * HH,
                                  ptx::desc_add(aq, ii * ATILE + ks * 256),
                                  ptx::desc_add(bq, (QM ? ii * HPG * HPG * 2 : 0) + v * (HH * HPG * 2) + ks * 256),
                                  idesc_mix, ks > 0);
          if (ptx::elect_one()) ptx::mma_commit(bar_D + sg);
          __syncwarp();
        }
    };
    if (warp == mma_warp) {
      int scnt[2] = {0, 0}, sidx = 0;
      // S^T = K Q^T of one key tile into S buffer buf, K jobs from job0 of
      // the pass-A (ring_a) or pass-B ring
      auto qk = [&](int buf, int job0, bool ring_a) {
        uint64_t *full = ring_a ? bar_afull : bar_kfull, *freeb = ring_a ? bar_afree : bar_kfree;
        const int nslot = ring_a ? NKA : NSK;
        if (scnt[buf] >= 1) wait_u(bar_Sfree + buf, (scnt[buf] - 1) & 1, ERR_TIMEOUT_S);
        ++scnt[buf];
        ++sidx;
        if (!ok) return;
        ptx::tc_fence_after();
        for (int h0 = 0, job = job0; h0 < HPG; h0 += HJ, job += HJ) {
          wait_jobs(job, full, nslot);
          if (!ok) return;
          uint64_t ka[HJ], qa[HJ];
          uint32_t dd[HJ];
#pragma unroll
          for (int hh = 0; hh < HJ; ++hh) {
            const int h = (h0 + hh + hrot) % HPG;
            ka[hh] = ptx::desc_add(dsm, kslot_off(ring_a, (job + hh) % nslot));
            qa[hh] = ptx::desc_add(ka[hh], KJOB);  // Q rows of head h follow its K tile
            dd[hh] = tbase + (static_cast<uint32_t>(16 * (h / HH)) << 16) + s_col(buf) + (h % HH) * BM;
          }
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)
#pragma unroll
            for (int hh = 0; hh < HJ; ++hh)
              if (ptx::elect_one())
                ptx::mma_f16_ss(dd[hh], ptx::desc_add(ka[hh], (ks >> 2) * (KJOB / 2) + (ks & 3) * 32),
                                ptx::desc_add(qa[hh], (ks >> 2) * (BM * 128) + (ks & 3) * 32), idesc_qk, ks > 0);
          free_jobs(job, freeb, nslot);
        }
        if (ptx::elect_one()) ptx::mma_commit(bar_S + buf);
        __syncwarp();
      };
      // pass A: S tiles alternate between the two buffers; pass B: buffer 0
      for (int kt = 0; kt < nkt && ok; ++kt) qk(kt & 1, kt * HPG, true);
      for (int kt = 0; kt < nkt && ok; ++kt) qk(0, kt * HPG, false);
    } else if (warp == mix_warp) {
      for (int kt = 0; kt < nkt && ok; ++kt) mixes(0, kt);
      for (int kt = 0; kt < nkt && ok; ++kt) {
        mixes(0, nkt + 2 * kt);
        mixes(1, nkt + 2 * kt + 1);
      }
    } else {
      // O^T += V^T P'^T per key tile of pass B
      for (int kt = 0; kt < nkt && ok; ++kt) {
        wait_u(bar_P, kt & 1, ERR_TIMEOUT_P);
        if (!ok) break;
        ptx::tc_fence_after();
        const int nks = (kt == nkt - 1 ? rlast : KT) / 16;
        const int job0 = kt * HPG;
        for (int h0 = 0, job = job0; h0 < HPG; h0 += HJ, job += HJ) {
          wait_jobs(job, bar_vfull, NSV);
          if (!ok) break;
          uint64_t va[HJ], pa[HJ];
          uint32_t dd[HJ];
#pragma unroll
          for (int hh = 0; hh < HJ; ++hh) {
            const int h = (h0 + hh + hrot) % HPG;
            va[hh] = ptx::desc_add(dv0, ((job + hh) % NSV) * KJOB);
            pa[hh] = ptx::desc_add(dp0, h * PHEAD);
            dd[hh] = tbase + O_COL + h * BM;
          }
#pragma unroll
          for (int ks = 0; ks < KT / 16; ++ks) {
            if (ks < nks) {
#pragma unroll
              for (int hh = 0; hh < HJ; ++hh)
#pragma unroll
                for (int c = 0; c < 2; ++c)
                  if (ptx::elect_one())
                    ptx::mma_f16_ss(dd[hh] + (static_cast<uint32_t>(16 * c) << 16),
                                    ptx::desc_add(va[hh], c * (KJOB / 2) + ks * 2048),
                                    ptx::desc_add(pa[hh], ks * (2 * BM * 16)), idesc_pv, (kt > 0 || ks > 0));
            }
          }
          free_jobs(job, bar_vfree, NSV);
        }
        if (ptx::elect_one()) ptx::mma_commit(bar_Pfree);
        __syncwarp();
      }
      if (ptx::elect_one()) ptx::mma_commit(bar_O);
      __syncwarp();
    }
  } else {
    // ============================================================ compose warps
    const int qtr = warp & 3, cs = warp >> 2;
    const int u = lane >> 4, r16 = lane & 15;
    const int key_local = 16 * qtr + r16;
    const int ctid = threadIdx.x;
    const float sl2e = p.scale * kLog2e;
    const uint32_t tl = tbase + (static_cast<uint32_t>(32 * qtr) << 16);
    unsigned char *atile = smem + geo.a_off;
    unsigned char *ptile = smem + geo.p_off;

    // ---- static mix operands (fp16, K-major, no swizzle) and per-query records
    // (with QM one operand per (set, query): the static mix plus that query's
    // off-diagonal qmat entries; their diagonal joins the fp32 gates below)
    constexpr int NB = QM ? BM : 1;
    for (int idx = ctid; idx < 2 * NB * HPG * HPG; idx += 32 * NCW) {
      const int set = idx / (NB * HPG * HPG), i = (idx / (HPG * HPG)) % NB, rem = idx % (HPG * HPG);
      const int hout = rem / HPG, kin = rem % HPG;  // B[n][k] of output half hout / HH
      const TermPtrs &tm = set ? p.post : p.pre;
      float wv = (kin == hout || !tm.w) ? 0.f : tm.w[((int64_t)g * HPG + kin) * HPG + hout];
      if (QM && kin != hout) wv += qmat_at<E>(tm, b, q0 + i, T, H, HPG, hbase, kin, hout);
      const int v = hout / HH, n = hout % HH;
      __half *dst = reinterpret_cast<__half *>(smem + geo.bm_off + (set * NB + i) * (HPG * HPG * 2) +
                                               v * (HH * HPG * 2) + ((n / 8) * KB + kin / 8) * 128 + (n % 8) * 16 +
                                               (kin % 8) * 2);
      *dst = __float2half_rn(wv);
    }
    for (int idx = ctid; idx < 2 * BM * recf; idx += 32 * NCW) {
      const int set = idx / (BM * recf), rem = idx % (BM * recf);
      const int i = rem / recf, j = rem % recf;
      const TermPtrs &tm = set ? p.post : p.pre;
      const int t = q0 + i;
      float val = 0.f;
      if (t < T) {
        const int64_t tok = (int64_t)b * T + t;
        if (j < HPG) {
          val = (tm.identity ? 1.f : 0.f) + (tm.w ? tm.w[((int64_t)g * HPG + j) * HPG + j] : 0.f) +
                (tm.qdd ? ld_w<E>(tm.qdd, tok * H + hbase + j) : 0.f) +
                (QM ? qmat_at<E>(tm, b, t, T, H, HPG, hbase, j, j) : 0.f);
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
    ptx::fence_proxy_async_smem();
    ptx::named_bar_sync(1, 32 * NCW);

    bool ok = true;
    auto wait_or_fail = [&](uint64_t *bar, int parity, int code) {
      if (ok && !ptx::mbar_wait(bar, parity, WAIT)) {
        ok = false;
        record_err(p, code);
      }
    };
    auto arrive = [&](uint64_t *bar) {
      ptx::fence_proxy_async_smem();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar);
    };
    auto valid = [&](int s, int t) {
      return s <= t && (p.window <= 0 || t - s < p.window) && t < T;
    };

    // load S (this thread's key, its lane half's heads) for NQG queries
    auto load_s = [&](int sbuf, int i0, float (&a)[HH][NQG]) {
#pragma unroll
      for (int j = 0; j < HH; ++j) ptx::tmem_ld<NQG>(tl + s_col(sbuf) + j * BM + i0, a[j]);
    };
    // rank-R reductions over all HPG heads (two lane halves) and the mix operand rows
    auto reduce_and_stage = [&](const KeyW<HH, R> &kw, int set, int i0, const float (&a)[HH][NQG],
                                float (&aq)[NQG][R], float (&ak)[NQG][R]) {
      const float *rb = rec + (set * BM + i0) * recf;
#pragma unroll
      for (int i = 0; i < NQG; ++i)
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float sq = 0.f;
#pragma unroll
          for (int j = 0; j < HH; ++j) sq = fmaf(rb[i * recf + HPG + (HH * u + j) * R + r], a[j][i], sq);
          aq[i][r] = sq;
          float sk = 0.f;
#pragma unroll
          for (int j = 0; j < HH; ++j) sk = fmaf(unpack_e<E>(kw.w1, j * R + r), a[j][i], sk);
          ak[i][r] = sk;
        }
#pragma unroll
      for (int i = 0; i < NQG; ++i)
#pragma unroll
        for (int r = 0; r < R; ++r) {
          aq[i][r] += __shfl_xor_sync(0xffffffffu, aq[i][r], 16);
          ak[i][r] += __shfl_xor_sync(0xffffffffu, ak[i][r], 16);
        }
#pragma unroll
      for (int i = 0; i < NQG; ++i) {
        unsigned char *row = atile + (i0 + i) * ATILE + (key_local >> 3) * (KB * 128) + (key_local & 7) * 16;
#pragma unroll
        for (int kb = 0; kb < HH / 8; ++kb) {
          uint4 v;
          v.x = pack_h2(a[kb * 8 + 0][i], a[kb * 8 + 1][i]);
          v.y = pack_h2(a[kb * 8 + 2][i], a[kb * 8 + 3][i]);
          v.z = pack_h2(a[kb * 8 + 4][i], a[kb * 8 + 5][i]);
          v.w = pack_h2(a[kb * 8 + 6][i], a[kb * 8 + 7][i]);
          *reinterpret_cast<uint4 *>(row + (u * (HH / 8) + kb) * 128) = v;
        }
      }
    };
    // composed values x = mix (TMEM D) + diagonal gates * a + rank-R expansions
    auto finish = [&](const KeyW<HH, R> &kw, int set, int i0, const float (&dm)[NQG][HH],
                      const float (&a)[HH][NQG], const float (&aq)[NQG][R], const float (&ak)[NQG][R],
                      float (&x)[HH][NQG]) {
      const float *rb = rec + (set * BM + i0) * recf;
#pragma unroll
      for (int j = 0; j < HH; ++j) {
        const float kd = unpack_e<E>(kw.dd, j);
        float k2[R];
#pragma unroll
        for (int r = 0; r < R; ++r) k2[r] = unpack_e<E>(kw.w2, r * HH + j);
#pragma unroll
        for (int i = 0; i < NQG; ++i) {
          float xv = fmaf(rb[i * recf + HH * u + j] + kd, a[j][i], dm[i][j]);
#pragma unroll
          for (int r = 0; r < R; ++r)
            xv = fmaf(rb[i * recf + HPG + HPG * R + r * HPG + HH * u + j], aq[i][r], fmaf(k2[r], ak[i][r], xv));
          x[j][i] = xv;
        }
      }
    };
    auto load_d = [&](int i0, float (&dm)[NQG][HH]) {
#pragma unroll
      for (int i = 0; i < NQG; ++i) ptx::tmem_ld<HH>(tl + D_COL + (i0 + i) * HH, dm[i]);
    };

    int scnt[2] = {0, 0};  // uses of each S buffer so far (barrier phases)
    float m_run[NSG][2], l_run[NSG][2];
#pragma unroll
    for (int k = 0; k < NSG; ++k) { m_run[k][0] = m_run[k][1] = -INFINITY; l_run[k][0] = l_run[k][1] = 0.f; }

    // ============================== pass A: statistics of the composed logits
    for (int kt = 0; kt < nkt; ++kt) {
      const int s = k_lo + kt * KT + key_local;
      const bool key_ok = s < slen;
      const int64_t tok = (int64_t)b * T + s;
      KeyW<HH, R> kwp;
      load_keyw<E, HH, R>(kwp, p.pre, tok, H, hbase + HH * u, key_ok);
      const int sbuf = kt & 1;
      wait_or_fail(bar_S + sbuf, scnt[sbuf] & 1, ERR_TIMEOUT_S);
      ptx::tc_fence_after();
      float aq[NSG][NQG][R], ak[NSG][NQG][R];
#pragma unroll
      for (int sgl = 0; sgl < NSG; ++sgl) {
        const int i0 = (cs * NSG + sgl) * NQG;
        float a[HH][NQG];
        load_s(sbuf, i0, a);
        ptx::tmem_wait_ld();
        reduce_and_stage(kwp, 0, i0, a, aq[sgl], ak[sgl]);
        arrive(bar_A + cs * NSG + sgl);
      }
#pragma unroll
      for (int sgl = 0; sgl < NSG; ++sgl) {
        const int sg = cs * NSG + sgl, i0 = sg * NQG;
        wait_or_fail(bar_D + sg, kt & 1, ERR_TIMEOUT_P);
        ptx::tc_fence_after();
        float dm[NQG][HH], a[HH][NQG], x[HH][NQG];
        load_d(i0, dm);
        load_s(sbuf, i0, a);
        ptx::tmem_wait_ld();
        finish(kwp, 0, i0, dm, a, aq[sgl], ak[sgl], x);
        // masked max / exp / transposed sum over the 16 keys of this lane half
        float e[32], mt[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int j = c / NQG, i = c % NQG;
          const float v = (key_ok && valid(s, q0 + i0 + i)) ? x[j][i] : -INFINITY;
          const float m0 = ptx::warp_max(u == 0 ? v : -INFINITY);
          const float m1 = ptx::warp_max(u == 1 ? v : -INFINITY);
          const float mw = u ? m1 : m0;
          if (r16 == (c >> 1)) mt[c & 1] = mw;
          e[c] = exp2f((v - (mw == -INFINITY ? 0.f : mw)) * sl2e);
        }
#pragma unroll
        for (int off = 8, cnt = 32; off >= 1; off >>= 1, cnt >>= 1) {
          const bool upper = (lane & off) != 0;
#pragma unroll
          for (int jj = 0; jj < cnt / 2; ++jj) {
            const float send = upper ? e[jj] : e[jj + cnt / 2];
            const float keep = upper ? e[jj + cnt / 2] : e[jj];
            e[jj] = keep + __shfl_xor_sync(0xffffffffu, send, off);
          }
        }
#pragma unroll
        for (int k = 0; k < 2; ++k)
          if (mt[k] != -INFINITY) {
            const float mn = fmaxf(m_run[sgl][k], mt[k]);
            l_run[sgl][k] = (m_run[sgl][k] == -INFINITY ? 0.f : l_run[sgl][k] * exp2f((m_run[sgl][k] - mn) * sl2e)) +
                            e[k] * exp2f((mt[k] - mn) * sl2e);
            m_run[sgl][k] = mn;
          }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_Sfree + sbuf);
      ++scnt[sbuf];
    }
    // ---- combine the lane quarters
#pragma unroll
    for (int sgl = 0; sgl < NSG; ++sgl)
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int c = 2 * r16 + k, j = c / NQG, i = c % NQG;
        const int col = (HH * u + j) * BM + (cs * NSG + sgl) * NQG + i;
        redm[qtr * NCOL + col] = m_run[sgl][k];
        reds[qtr * NCOL + col] = l_run[sgl][k];
      }
    ptx::named_bar_sync(1, 32 * NCW);
    for (int jc = ctid; jc < NCOL; jc += 32 * NCW) {
      float m = -INFINITY;
      for (int q = 0; q < 4; ++q) m = fmaxf(m, redm[q * NCOL + jc]);
      float l = 0.f;
      for (int q = 0; q < 4; ++q) {
        const float mq = redm[q * NCOL + jc];
        if (mq != -INFINITY) l += reds[q * NCOL + jc] * exp2f((mq - m) * sl2e);
      }
      mval[jc] = m == -INFINITY ? 0.f : m * sl2e;
      linv[jc] = l > 0.f ? 1.f / l : 0.f;
    }
    ptx::named_bar_sync(1, 32 * NCW);

    // ============================== pass B: probabilities, post mix, P'V
    for (int kt = 0; kt < nkt; ++kt) {
      const int s = k_lo + kt * KT + key_local;
      const bool key_ok = s < slen;
      const int64_t tok = (int64_t)b * T + s;
      const int rpre = nkt + 2 * kt, rpost = rpre + 1;
      KeyW<HH, R> kwp, kwq;
      load_keyw<E, HH, R>(kwp, p.pre, tok, H, hbase + HH * u, key_ok);
      const int sbuf = 0;
      wait_or_fail(bar_S + sbuf, scnt[sbuf] & 1, ERR_TIMEOUT_S);
      ptx::tc_fence_after();
      float aq[NSG][NQG][R], ak[NSG][NQG][R];
#pragma unroll
      for (int sgl = 0; sgl < NSG; ++sgl) {
        const int i0 = (cs * NSG + sgl) * NQG;
        float a[HH][NQG];
        load_s(sbuf, i0, a);
        ptx::tmem_wait_ld();
        reduce_and_stage(kwp, 0, i0, a, aq[sgl], ak[sgl]);
        arrive(bar_A + cs * NSG + sgl);
      }
      load_keyw<E, HH, R>(kwq, p.post, tok, H, hbase + HH * u, key_ok);
      float pr[NSG][HH][NQG], pq[NSG][NQG][R], pk[NSG][NQG][R];
#pragma unroll
      for (int sgl = 0; sgl < NSG; ++sgl) {
        const int sg = cs * NSG + sgl, i0 = sg * NQG;
        wait_or_fail(bar_D + sg, rpre & 1, ERR_TIMEOUT_P);
        ptx::tc_fence_after();
        float dm[NQG][HH], a[HH][NQG], x[HH][NQG];
        load_d(i0, dm);
        load_s(sbuf, i0, a);
        ptx::tmem_wait_ld();
        finish(kwp, 0, i0, dm, a, aq[sgl], ak[sgl], x);
#pragma unroll
        for (int j = 0; j < HH; ++j)
#pragma unroll
          for (int i = 0; i < NQG; ++i) {
            const int col = (HH * u + j) * BM + i0 + i;
            pr[sgl][j][i] = (key_ok && valid(s, q0 + i0 + i)) ? exp2f(fmaf(x[j][i], sl2e, -mval[col])) * linv[col]
                                                             : 0.f;
          }
        reduce_and_stage(kwq, 1, i0, pr[sgl], pq[sgl], pk[sgl]);
        arrive(bar_A + sg);
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_Sfree + sbuf);
      ++scnt[sbuf];
      if (kt >= 1) wait_or_fail(bar_Pfree, (kt - 1) & 1, ERR_TIMEOUT_P);
#pragma unroll
      for (int sgl = 0; sgl < NSG; ++sgl) {
        const int sg = cs * NSG + sgl, i0 = sg * NQG;
        wait_or_fail(bar_D + sg, rpost & 1, ERR_TIMEOUT_P);
        ptx::tc_fence_after();
        float dm[NQG][HH], x[HH][NQG];
        load_d(i0, dm);
        ptx::tmem_wait_ld();
        finish(kwq, 1, i0, dm, pr[sgl], pq[sgl], pk[sgl], x);
        unsigned char *prow = ptile + (key_local & 7) * 16 + (key_local >> 3) * (BM * 16);
#pragma unroll
        for (int j = 0; j < HH; ++j)
#pragma unroll
          for (int i = 0; i < NQG; i += 2) {
            const int qi = i0 + i;
            *reinterpret_cast<uint32_t *>(prow + (HH * u + j) * PHEAD + (qi >> 3) * 128 + (qi & 7) * 2) =
                pack_e2<E>(x[j][i], x[j][i + 1]);
          }
      }
      arrive(bar_P);
    }

    // ============================== epilogue: O^T -> SMEM [head][d half][query][64 d] -> TMA store
    wait_or_fail(bar_O, 0, ERR_TIMEOUT_O);
    ptx::tc_fence_after();
    unsigned char *stage = smem;  // pool base: every MMA has completed
    const int d = 64 * u + 16 * qtr + r16;
    if (ok) {
#pragma unroll 1
      for (int h = cs; h < HPG; h += 2) {
        float v[BM];
        ptx::tmem_ld<BM>(tl + O_COL + h * BM, v);
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

template <typename E, int HPG, int R, bool QM>
static cudaError_t launch_t(const dc_attn_params &p, cudaStream_t st) {
  using SH = Shape<HPG, QM>;
  const GeoM geo = make_geo_m<HPG, R, QM>();
  const size_t smem = geo.total + 1024;
  const int64_t sb = (int64_t)p.T * p.H * D, st_ = (int64_t)p.H * D, sh = D;
  CUtensorMap mq, mk, mv, mo;
  if (!make_map5(&mq, p.q, p.dtype, p.B, p.T, p.H, SH::BM, 1, sb, st_, sh) ||
      !make_map5(&mk, p.k, p.dtype, p.B, p.T, p.H, KT, 1, sb, st_, sh) ||
      !make_map5(&mv, p.v, p.dtype, p.B, p.T, p.H, KT, 1, sb, st_, sh) ||
      !make_map(&mo, p.out, p.dtype, p.B, p.T, p.H, SH::BM, p.out_sb, p.out_st, p.out_sh, false))
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
  auto kern = dc_tcm_kernel<E, HPG, R, QM>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((p.T + SH::BM - 1) / SH::BM, p.B * p.G);
  kern<<<grid, 32 * (NCW + 4), smem, st>>>(mq, mk, mv, mo, tp);
  return cudaGetLastError();
}

template <typename E, int HPG>
static cudaError_t launch_h(const dc_attn_params &p, cudaStream_t st) {
  if (p.pre.qmat || p.post.qmat)
    return p.R <= 1 ? launch_t<E, HPG, 1, true>(p, st) : launch_t<E, HPG, 2, true>(p, st);
  return p.R <= 1 ? launch_t<E, HPG, 1, false>(p, st) : launch_t<E, HPG, 2, false>(p, st);
}

template <typename E>
static cudaError_t launch_e(const dc_attn_params &p, cudaStream_t st) {
  return p.H / p.G == 32 ? launch_h<E, 32>(p, st) : launch_h<E, 16>(p, st);
}

}  // namespace tcm

bool tcm_supports(const dc_attn_params &p, std::string *why) {
  auto no = [&](const char *m) { if (why) *why = m; return false; };
  if (p.D != 128) return no("D must be 128");
  if (p.G <= 0 || (p.H / p.G != 16 && p.H / p.G != 32)) return no("heads per group must be 16 or 32");
  if (p.R > 2) return no("rank R > 2");
  if (!(p.scale > 0.f)) return no("non-positive softmax scale");
  auto al = [](const void *x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  if (!al(p.q) || !al(p.k) || !al(p.v) || !al(p.out)) return no("q, k, v, out must be 16-byte aligned");
  if (p.out_sb % 8 || p.out_st % 8 || p.out_sh % 8) return no("output strides must be multiples of 8 elements");
  if (p.H % 8) return no("H must be a multiple of 8");
  for (const dc_terms *t : {&p.pre, &p.post}) {
    for (const void *w : {t->kw1, t->kw2, t->kdd})
      if (w && !al(w)) return no("key-wise weights must be 16-byte aligned");
    if ((t->kw1 == nullptr) != (t->kw2 == nullptr)) return no("kw1 and kw2 must be given together");
  }
  return true;
}

cudaError_t launch_tcm(const dc_attn_params &p, cudaStream_t st) {
  if (p.dtype == DC_DTYPE_BF16) return tcm::launch_e<__nv_bfloat16>(p, st);
  return tcm::launch_e<__half>(p, st);
}

}  // namespace dcattn
