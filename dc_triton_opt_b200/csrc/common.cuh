// Shared device helpers for the DC-attention kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/dc_attn.h"

namespace dcattn {

template <typename E> __device__ __forceinline__ float to_f(E x);
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }

template <typename E> __device__ __forceinline__ E from_f(float x);
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

// Load one element of a per-token weight tensor through the read-only path.
template <typename E>
__device__ __forceinline__ float ldw(const void *base, int64_t idx) {
  return to_f<E>(__ldg(reinterpret_cast<const E *>(base) + idx));
}

constexpr float kLog2e = 1.4426950408889634f;

// Device-side copy of one composition term set.
struct TermsDev {
  int identity;
  const float *w;
  const void *qw1, *qw2, *kw1, *kw2, *qdd, *kdd, *qmat;
};

struct ParamsDev {
  int B, T, H, D, G, R, HPG;
  int window;  // <= 0: full causal
  float scale;
  const void *q, *k, *v;
  void *out;
  int64_t out_sb, out_st, out_sh;
  const int32_t *seq_lens;
  int32_t *err_flag;
  TermsDev pre, post;
};

inline TermsDev to_dev(const dc_terms &t) {
  TermsDev d;
  d.identity = t.identity;
  d.w = t.w;
  d.qw1 = t.qw1; d.qw2 = t.qw2; d.kw1 = t.kw1; d.kw2 = t.kw2;
  d.qdd = t.qdd; d.kdd = t.kdd; d.qmat = t.qmat;
  return d;
}

inline ParamsDev to_dev(const dc_attn_params &p) {
  ParamsDev d;
  d.B = p.B; d.T = p.T; d.H = p.H; d.D = p.D; d.G = p.G; d.R = p.R;
  d.HPG = p.H / p.G;
  d.window = p.window; d.scale = p.scale;
  d.q = p.q; d.k = p.k; d.v = p.v; d.out = p.out;
  d.out_sb = p.out_sb; d.out_st = p.out_st; d.out_sh = p.out_sh;
  d.seq_lens = p.seq_lens; d.err_flag = p.err_flag;
  d.pre = to_dev(p.pre); d.post = to_dev(p.post);
  return d;
}

}  // namespace dcattn
