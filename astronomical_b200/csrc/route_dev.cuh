// route_dev.cuh -- per-token routing (softmax over E, top-K, renormalisation)
// as a warp-level device function, shared by the route kernel and the fused
// decode kernel.  Semantics: qwen3_5_moe_route_experts
// (qwen3_5_moe/model/routing.rs:16-49); reduction order and tie policy as in
// route.cu's header comment.
#pragma once

#include "common.cuh"

namespace astro {

template <typename T> struct RouteKey;
// 16-bit types: probabilities are >= 0, so their bit patterns order like the
// values; key = (bits << 16) | (0xffff - id) and max gives (value desc, id asc).
template <> struct RouteKey<__nv_bfloat16> {
  static ASTRO_DEVINL uint32_t bits(float p) { return f32_to_bf16(p); }
  static ASTRO_DEVINL float value(uint32_t b) { return bf16_to_f32((uint16_t)b); }
};
template <> struct RouteKey<__half> {
  static ASTRO_DEVINL uint32_t bits(float p) { return __half_as_ushort(__float2half_rn(p)); }
  static ASTRO_DEVINL float value(uint32_t b) { return __half2float(__ushort_as_half((uint16_t)b)); }
};

// Routes one token with the calling warp: `row` holds its E logits; lane k < K
// writes winner k to ids[k] / scores[k] (any address space).
template <typename T, int CMAX>
ASTRO_DEVINL void route_token(const T* row, int E, int K, int normalize, uint32_t* ids,
                              T* scores) {
  const int lane = threadIdx.x & 31;
  const int C = (E + 31) >> 5;
  const int i0 = lane * C;

  float v[CMAX];
  float mx = -INFINITY;
#pragma unroll
  for (int c = 0; c < CMAX; ++c) {
    const int i = i0 + c;
    v[c] = (c < C && i < E) ? Num<T>::load(row, i) : -INFINITY;
    mx = (v[c] > mx) ? v[c] : mx;
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, mx, m);
    mx = (o > mx) ? o : mx;
  }
  float part = 0.0f;
#pragma unroll
  for (int c = 0; c < CMAX; ++c) {
    const int i = i0 + c;
    if (c < C && i < E) {
      v[c] = expf_cw(__fsub_rn(v[c], mx));
      part = __fadd_rn(part, v[c]);
    }
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, m));
  const float inv = __fdiv_rn(1.0f, part);

  // probabilities rounded to the logits dtype; top-K selection
  uint32_t key[CMAX];
#pragma unroll
  for (int c = 0; c < CMAX; ++c) {
    const int i = i0 + c;
    const bool valid = (c < C && i < E);
    const float p = Num<T>::round(__fmul_rn(v[c], inv));
    if constexpr (sizeof(T) == 2) {
      key[c] = valid ? ((RouteKey<T>::bits(p) << 16) | (0xffffu - (uint32_t)i)) : 0u;
    } else {
      v[c] = valid ? p : -1.0f;
      key[c] = valid ? 1u : 0u;  // liveness only
    }
  }

  // Up to 8 keys a lane (E <= 256): the lane's keys are sorted once, descending
  // (bitonic network), so a selection round is one warp max over the lanes'
  // first keys and a shift in the winning lane; keys are unique (they carry the
  // expert id), so the winners and their order are those of a max over all keys.
  constexpr bool kSortedKeys = sizeof(T) == 2 && CMAX <= 8;
  if constexpr (kSortedKeys) {
#pragma unroll
    for (int kk = 2; kk <= CMAX; kk <<= 1) {
#pragma unroll
      for (int j = kk >> 1; j >= 1; j >>= 1) {
#pragma unroll
        for (int i = 0; i < CMAX; ++i) {
          const int l = i ^ j;
          if (l > i) {
            const uint32_t a = key[i], b = key[l];
            const bool desc = (i & kk) == 0;
            key[i] = desc ? (a > b ? a : b) : (a < b ? a : b);
            key[l] = desc ? (a > b ? b : a) : (a < b ? b : a);
          }
        }
      }
    }
  }

  float sel_val = 0.0f;  // lane k keeps winner k
  uint32_t sel_id = 0;
  float sum_sel = 0.0f;
  for (int k = 0; k < K; ++k) {
    uint32_t wid;
    float wval;
    if constexpr (kSortedKeys) {
      const uint32_t best = __reduce_max_sync(0xffffffffu, key[0]);
      wid = 0xffffu - (best & 0xffffu);
      wval = RouteKey<T>::value(best >> 16);
      const bool won = key[0] == best;
#pragma unroll
      for (int c = 0; c + 1 < CMAX; ++c) key[c] = won ? key[c + 1] : key[c];
      if (won) key[CMAX - 1] = 0u;
    } else if constexpr (sizeof(T) == 2) {
      uint32_t best = 0;
#pragma unroll
      for (int c = 0; c < CMAX; ++c) best = (key[c] > best) ? key[c] : best;
      best = __reduce_max_sync(0xffffffffu, best);
      wid = 0xffffu - (best & 0xffffu);
      wval = RouteKey<T>::value(best >> 16);
#pragma unroll
      for (int c = 0; c < CMAX; ++c)
        if (key[c] == best) key[c] = 0u;
    } else {
      // fp32 probabilities: (value desc, id asc) with a 64-bit key
      uint64_t best = 0;
#pragma unroll
      for (int c = 0; c < CMAX; ++c) {
        if (key[c]) {
          const uint64_t kk = ((uint64_t)__float_as_uint(v[c]) << 32) |
                              (uint64_t)(0xffffffffu - (uint32_t)(i0 + c));
          best = (kk > best) ? kk : best;
        }
      }
#pragma unroll
      for (int m = 16; m >= 1; m >>= 1) {
        const uint64_t o = __shfl_xor_sync(0xffffffffu, best, m);
        best = (o > best) ? o : best;
      }
      wid = 0xffffffffu - (uint32_t)(best & 0xffffffffu);
      wval = __uint_as_float((uint32_t)(best >> 32));
#pragma unroll
      for (int c = 0; c < CMAX; ++c)
        if (key[c] && (uint32_t)(i0 + c) == wid) key[c] = 0u;
    }
    if (lane == k) {
      sel_val = wval;
      sel_id = wid;
    }
    sum_sel = __fadd_rn(sum_sel, wval);
  }
  if (lane < K) {
    float s = sel_val;
    if (normalize) s = Num<T>::round(__fdiv_rn(sel_val, Num<T>::round(sum_sel)));
    ids[lane] = sel_id;
    Num<T>::store(scores, lane, s);
  }
}


// fp32 -> uint32 whose unsigned order is the IEEE total order (total_cmp)
ASTRO_DEVINL uint32_t ordered_bits(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Laguna routing of one token with the calling warp (route_laguna_experts,
// laguna/moe/router.rs:11-60; CPU owner laguna/moe/router_selection.rs:47-107):
// score = sigmoid(softcap > 0 ? softcap * tanh(logit / softcap) : logit) in fp32,
// selection = score + bias[e] (bias may be null), the K largest selections by
// (value desc, id asc; IEEE total order), each winner's original score, and with
// `normalize` the scores divided by their sum (in slot order) when it is > 0.
// Lane k < K writes winner k to ids[k] / scores[k].
template <typename T, int CMAX>
ASTRO_DEVINL void route_token_laguna(const T* row, int E, int K, float softcap, const float* bias,
                                     int normalize, uint32_t* ids, float* scores) {
  const int lane = threadIdx.x & 31;
  const int C = (E + 31) >> 5;
  const int i0 = lane * C;
  float orig[CMAX];
  uint64_t key[CMAX];
#pragma unroll
  for (int c = 0; c < CMAX; ++c) {
    const int i = i0 + c;
    const bool valid = c < C && i < E;
    float l = valid ? Num<T>::load(row, i) : 0.0f;
    if (softcap > 0.0f) l = __fmul_rn(tanh_cw(__fdiv_rn(l, softcap)), softcap);
    const float sc = sigmoid_plain(l);
    const float sel = bias ? __fadd_rn(sc, bias[valid ? i : 0]) : sc;
    orig[c] = sc;
    key[c] = valid ? (((uint64_t)ordered_bits(sel) << 32) | (uint64_t)(0xffffffffu - (uint32_t)i)) : 0ull;
  }
  float sel_score = 0.0f;
  uint32_t sel_id = 0;
  float sum = 0.0f;
  for (int k = 0; k < K; ++k) {
    uint64_t best = 0;
#pragma unroll
    for (int c = 0; c < CMAX; ++c) best = key[c] > best ? key[c] : best;
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      const uint64_t o = __shfl_xor_sync(0xffffffffu, best, m);
      best = o > best ? o : best;
    }
    const uint32_t wid = 0xffffffffu - (uint32_t)(best & 0xffffffffu);
    float mine = 0.0f;
#pragma unroll
    for (int c = 0; c < CMAX; ++c)
      if (key[c] == best) {
        mine = orig[c];
        key[c] = 0ull;
      }
    const float w = __shfl_sync(0xffffffffu, mine, (int)(wid / (uint32_t)C));
    if (lane == k) {
      sel_score = w;
      sel_id = wid;
    }
    sum = __fadd_rn(sum, w);
  }
  if (lane < K) {
    ids[lane] = sel_id;
    scores[lane] = (normalize && sum > 0.0f) ? __fdiv_rn(sel_score, sum) : sel_score;
  }
}

}  // namespace astro
