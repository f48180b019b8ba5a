// Device helpers shared by the single-launch frame kernels (tile and pair):
// bf16 packing, GELU-tanh, the TMEM position layout, and the warp-per-row
// sampler that finishes the top-k select from the constrained logits and row
// maximum a head epilogue leaves (same sampling contract as sample_block in
// sampling.cuh: local_ar_plugins.cu:1211-1370).
#pragma once

#include "common.cuh"
#include "frame_common.cuh"

namespace mtt {
namespace {

constexpr int kVocabChunks = kVocab / 8;  // 253 chunks of 8 values per row

__device__ __forceinline__ __nv_bfloat162 bf2_of(uint32_t w) { return *reinterpret_cast<const __nv_bfloat162*>(&w); }

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = __bfloat1622float2(h[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  return u;
}

// GELU, tanh form: tanh(u) = 1 - 2 / (exp(2u) + 1), with the fast exponential
// (error ~1e-6 relative before the result is rounded to bf16).
__device__ __forceinline__ float gelu_tanh(float v) {
  const float inner = 0.7978845608028654f * (v + 0.044715f * v * v * v);
  const float t = 1.0f - __fdividef(2.0f, __expf(2.0f * inner) + 1.0f);
  return 0.5f * v * (1.0f + t);
}

// TMEM column block of position j: even positions in blocks 0..7, odd in 8..15,
// so each part's positions are contiguous (four per 64-column load).
__device__ __forceinline__ int tmem_block(int j) { return 8 * (j & 1) + (j >> 1); }

constexpr uint32_t kKeyNegInf = 0x007fu;  // order key of bf16 -inf

// Order key of a bf16 bit pattern with -0 folded onto +0 (key order == float order).
__device__ __forceinline__ uint32_t sample_key(uint32_t b) {
  b = (b == 0x8000u) ? 0u : b;
  return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
}

// Constrained value of token t (bf16 bits): non-finite -> -inf (and flagged),
// forbidden specials / gated EOS -> -inf, finished -> EOS 0, others -inf.
__device__ __forceinline__ uint32_t constrain(uint32_t b, int t, bool unfinished, bool finished, bool forbid,
                                              bool& nonfinite) {
  if ((b & 0x7f80u) == 0x7f80u) {
    nonfinite = true;
    b = 0xff80u;
  }
  if (t >= kCodebook && (t != kEosId || unfinished || forbid)) b = 0xff80u;
  if (finished) b = (t == kEosId) ? 0u : 0xff80u;
  return b;
}

constexpr int kListCap = 512;  // candidate / eligible list capacity per row (u16 tokens)

struct Best {
  float score;
  int id;
};

__device__ __forceinline__ void keep_best(Best& b, float sc, int t) {
  if (sc > b.score || (sc == b.score && t < b.id)) {
    b.score = sc;
    b.id = t;
  }
}

__device__ __forceinline__ Best warp_best(Best b) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float os = __shfl_xor_sync(0xffffffffu, b.score, o);
    const int oi = __shfl_xor_sync(0xffffffffu, b.id, o);
    keep_best(b, os, oi);
  }
  return b;
}

// Philox-Gumbel scores of the tokens list[0, total), exact: with up to 128
// tokens every token is first scored with the library logf (within 1e-5 of
// the contract's correctly rounded Gumbel; scores stay within 1e-4), then
// only the tokens whose fast score is within kVerifyMargin of the best fast
// score are rescored with the correctly rounded log.  The exact winner's fast
// score is at least (best fast score - 2e-4), so it is always rescored: the
// result is the exact left-most argmax; when it is the only token within the
// margin it is the winner without rescoring.  Longer lists are scored exactly.
// Score with the contract's Gumbel (one copy of the double-precision log code).
__device__ __noinline__ float exact_score(float value, float temperature, uint32_t seed32, uint64_t offset) {
  return __fadd_rn(__fdiv_rn(value, temperature), clamped_gumbel(philox_uniform(seed32, offset)));
}

__device__ __forceinline__ void score_list(const uint16_t* list, uint32_t total, const uint16_t* vals, uint32_t seed32,
                                           uint64_t off64, float temperature, Best& b) {
  const int lane = threadIdx.x & 31;
  if (total <= 128) {
    float fs[4];
    float best_fast = -CUDART_INF_F;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      fs[j] = -CUDART_INF_F;
      const uint32_t e = lane + 32 * j;
      if (e < total) {
        const int t = list[e];
        const float u = philox_uniform(seed32, off64 + static_cast<uint64_t>(t));
        fs[j] = __fadd_rn(__fdiv_rn(bits2f(vals[t]), temperature), fast_gumbel(u));
        best_fast = fmaxf(best_fast, fs[j]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best_fast = fmaxf(best_fast, __shfl_xor_sync(0xffffffffu, best_fast, o));
    const float cut = best_fast - kVerifyMargin;
    uint32_t verify = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) verify |= (fs[j] >= cut ? 1u : 0u) << j;
    if (__reduce_add_sync(0xffffffffu, __popc(verify)) == 1) {
      // a single token within the margin: it is the exact winner (no other
      // token's exact score can reach it), and only the token is needed
      if (verify) {
        const int j = __ffs(verify) - 1;
        keep_best(b, fs[j], list[lane + 32 * j]);
      }
      return;
    }
    while (verify) {
      const int j = __ffs(verify) - 1;
      verify &= verify - 1;
      const int t = list[lane + 32 * j];
      keep_best(b, exact_score(bits2f(vals[t]), temperature, seed32, off64 + static_cast<uint64_t>(t)), t);
    }
  } else {
    for (uint32_t e = lane; e < total; e += 32) {
      const int t = list[e];
      keep_best(b, exact_score(bits2f(vals[t]), temperature, seed32, off64 + static_cast<uint64_t>(t)), t);
    }
  }
}


// bf16 value of an order key (the smallest key is -inf).
__device__ __forceinline__ __nv_bfloat16 key_value(uint32_t key) {
  return __ushort_as_bfloat16(static_cast<unsigned short>(key_bf16(key < kKeyNegInf ? kKeyNegInf : key)));
}

// Number of values >= v in a session's row (warp total): bf16x2 compares
// (-0 == +0, as in the float comparison the contract uses) summed in bf16x2.
__device__ __forceinline__ uint32_t count_ge(const uint16_t* vals, __nv_bfloat16 v) {
  const int lane = threadIdx.x & 31;
  const __nv_bfloat162 t2 = __bfloat162bfloat162(v);
  __nv_bfloat162 acc = __float2bfloat162_rn(0.f);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int ch = lane + 32 * i;
    if (ch < kVocabChunks) {
      const uint4 q = *reinterpret_cast<const uint4*>(vals + 8 * ch);
      acc = __hadd2(acc, __hge2(bf2_of(q.x), t2));
      acc = __hadd2(acc, __hge2(bf2_of(q.y), t2));
      acc = __hadd2(acc, __hge2(bf2_of(q.z), t2));
      acc = __hadd2(acc, __hge2(bf2_of(q.w), t2));
    }
  }
  const float2 f = __bfloat1622float2(acc);
  return __reduce_add_sync(0xffffffffu, static_cast<uint32_t>(f.x + f.y));
}

// The calling warp samples one session row from the constrained bf16 values
// and the row maximum a head epilogue left (same contract as sample_block in
// sampling.cuh).
// Top-k threshold (the k-th largest value, ties included), without atomics:
// one bf16x2 counting pass finds the smallest window of 32/64/128/256 key
// steps below the maximum that holds k values; the window's tokens form a
// candidate list whose distances below the maximum sit in registers, and a
// binary search over them gives the exact k-th largest.  Only eligible
// candidates are scored.  Rows whose window cannot be used (flat or very
// spread rows) take an exact binary search over the whole row instead.
// One session row at one position, as left by a head epilogue.
// bf16x2 guided logits of two adjacent tokens from the conditional and
// unconditional bf16x2 logits: bf16(bf16(c * s) + u * (1 - s)) per half, with
// the f32 add then the bf16 rounding (the plugin's two roundings).
__device__ __forceinline__ uint32_t guided_value2(uint32_t c2, uint32_t u2, float cfg_scale, float uncond_scale) {
  const float2 cf = __bfloat1622float2(bf2_of(c2));
  const float2 uf = __bfloat1622float2(bf2_of(u2));
  const float2 sc = __bfloat1622float2(__floats2bfloat162_rn(__fmul_rn(cf.x, cfg_scale), __fmul_rn(cf.y, cfg_scale)));
  const __nv_bfloat162 g = __floats2bfloat162_rn(__fadd_rn(sc.x, __fmul_rn(uf.x, uncond_scale)),
                                                 __fadd_rn(sc.y, __fmul_rn(uf.y, uncond_scale)));
  return *reinterpret_cast<const uint32_t*>(&g);
}

// Constrained values of tokens n, n + 1 (bf16x2); the slow path only for
// non-finite values, the special tokens and finished rows.
__device__ __forceinline__ uint32_t constrain2(uint32_t g, int n, uint32_t fl, bool& nonfinite) {
  const bool bad = ((g & 0x7f80u) == 0x7f80u) || ((g & 0x7f800000u) == 0x7f800000u);
  if (bad || n + 1 >= kCodebook || (fl & 2u)) {
    const bool u = fl & 1u, fin = fl & 2u, fb = fl & 4u;
    g = constrain(g & 0xffffu, n, u, fin, fb, nonfinite) | (constrain(g >> 16, n + 1, u, fin, fb, nonfinite) << 16);
  }
  return g;
}

__device__ __forceinline__ uint32_t pack2_rn(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

struct RowSample {
  const uint16_t* vals;  // 2024 constrained values (bf16 bits)
  uint32_t flags;        // bit 0 unfinished, bit 1 finished, bit 2 forbid_eos
  bool nonfinite;        // some guided logit of the row was NaN or infinite
  int64_t seed, counter;
};

// Order key of the row's maximum (bf16x2 max over the row, warp total).
__device__ __forceinline__ uint32_t row_max_key(const uint16_t* vals) {
  const int lane = threadIdx.x & 31;
  __nv_bfloat162 m2 = __bfloat162bfloat162(__ushort_as_bfloat16(static_cast<unsigned short>(0xff80u)));
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int ch = lane + 32 * i;
    if (ch < kVocabChunks) {
      const uint4 q = *reinterpret_cast<const uint4*>(vals + 8 * ch);
      m2 = __hmax2(m2, __hmax2(__hmax2(bf2_of(q.x), bf2_of(q.y)), __hmax2(bf2_of(q.z), bf2_of(q.w))));
    }
  }
  const uint32_t w = *reinterpret_cast<const uint32_t*>(&m2);
  const uint32_t k0 = sample_key(w & 0xffffu), k1 = sample_key(w >> 16);
  return __reduce_max_sync(0xffffffffu, k0 > k1 ? k0 : k1);
}

// Left-most token whose key is M (warp total).
__device__ __forceinline__ int row_first_key(const uint16_t* vals, uint32_t M) {
  const int lane = threadIdx.x & 31;
  int first = kVocab;
#pragma unroll
  for (int i = 7; i >= 0; --i) {
    const int ch = lane + 32 * i;
    if (ch < kVocabChunks) {
      const uint4 q = *reinterpret_cast<const uint4*>(vals + 8 * ch);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int e = 3; e >= 0; --e) {
        if (sample_key(w[e] >> 16) == M) first = 8 * ch + 2 * e + 1;
        if (sample_key(w[e] & 0xffffu) == M) first = 8 * ch + 2 * e;
      }
    }
  }
  return static_cast<int>(__reduce_min_sync(0xffffffffu, static_cast<uint32_t>(first)));
}

__device__ int sample_row(const RowSample& rs, const SamplingParams& prm, uint16_t* list, uint16_t* elig,
                          int* invalid_out) {
  const int lane = threadIdx.x & 31;
  const bool unfinished = rs.flags & 1u, finished = rs.flags & 2u, forbid = rs.flags & 4u;
  const int64_t seed = rs.seed;
  const int64_t counter = rs.counter;
  const bool nonfinite = rs.nonfinite;
  const uint32_t M = row_max_key(rs.vals);
  if (prm.argmax) {
    *invalid_out = (nonfinite || M == kKeyNegInf) ? 1 : 0;
    return M == kKeyNegInf ? 0 : row_first_key(rs.vals, M);
  }
  int invalid = (nonfinite || (unfinished && finished) || (finished && forbid)) ? 1 : 0;
  const bool seed_valid = seed >= 0 && static_cast<uint64_t>(seed) < (1ull << 32);
  const bool counter_valid = counter >= 0 && counter <= kMaxCounter;
  if (!seed_valid || !counter_valid) invalid = 1;
  if (finished) {  // only EOS (value 0) is finite: it is the only eligible token
    *invalid_out = invalid;
    return kEosId;
  }
  if (M == kKeyNegInf) {  // nothing finite
    *invalid_out = 1;
    return 0;
  }
  const uint32_t seed32 = seed_valid ? static_cast<uint32_t>(seed) : 0u;
  const uint64_t off64 = counter_valid ? static_cast<uint64_t>(counter) * kPhiloxStride : 0ull;
  const uint16_t* vals = rs.vals;
  const uint32_t kk = static_cast<uint32_t>(prm.top_k);

  // ---- pass 1: values within 32 / 64 / 128 / 256 key steps below the maximum
  __nv_bfloat162 lim[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) lim[j] = __bfloat162bfloat162(key_value(M + 1 < (32u << j) ? 0u : M + 1 - (32u << j)));
  __nv_bfloat162 acc[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) acc[j] = __float2bfloat162_rn(0.f);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int ch = lane + 32 * i;
    if (ch < kVocabChunks) {
      const uint4 q = *reinterpret_cast<const uint4*>(vals + 8 * ch);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int e = 0; e < 4; ++e)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[j] = __hadd2(acc[j], __hge2(bf2_of(w[e]), lim[j]));
    }
  }
  uint32_t mine4[4], tot[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f2 = __bfloat1622float2(acc[j]);
    mine4[j] = static_cast<uint32_t>(f2.x + f2.y);
    tot[j] = __reduce_add_sync(0xffffffffu, mine4[j]);
  }
  int win = 4;
#pragma unroll
  for (int j = 3; j >= 0; --j) win = tot[j] >= kk ? j : win;

  Best best{-CUDART_INF_F, kVocab};
  if (win < 4 && tot[win] <= static_cast<uint32_t>(kListCap)) {
    const __nv_bfloat162 limw = win == 0 ? lim[0] : (win == 1 ? lim[1] : (win == 2 ? lim[2] : lim[3]));
    const uint32_t mine = win == 0 ? mine4[0] : (win == 1 ? mine4[1] : (win == 2 ? mine4[2] : mine4[3]));
    const uint32_t n_cand = tot[win];
    uint32_t pos = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, pos, o);
      if (lane >= o) pos += y;
    }
    pos -= mine;
    // ---- pass 2: the window's tokens
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int ch = lane + 32 * i;
      if (ch < kVocabChunks) {
        const uint4 q = *reinterpret_cast<const uint4*>(vals + 8 * ch);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t m = __hge2_mask(bf2_of(w[e]), limw);
          if (m & 1u) list[pos] = static_cast<uint16_t>(8 * ch + 2 * e);
          pos += m & 1u;
          if (m >> 31) list[pos] = static_cast<uint16_t>(8 * ch + 2 * e + 1);
          pos += m >> 31;
        }
      }
    }
    __syncwarp();
    // ---- candidates' distances below the maximum, 16 per lane in registers
    uint32_t dist[kListCap / 32];
    uint16_t tokn[kListCap / 32];
#pragma unroll
    for (int m = 0; m < kListCap / 32; ++m) {
      const uint32_t e = lane + 32 * m;
      const int t = e < n_cand ? list[e] : 0;
      tokn[m] = static_cast<uint16_t>(t);
      dist[m] = e < n_cand ? M - sample_key(vals[t]) : 0xffffu;
    }
    // smallest d with count(dist <= d) >= k
    int lo = -1, hi = static_cast<int>((32u << win) - 1);
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      uint32_t cnt = 0;
#pragma unroll
      for (int m = 0; m < kListCap / 32; ++m) cnt += dist[m] <= static_cast<uint32_t>(mid);
      if (__reduce_add_sync(0xffffffffu, cnt) >= kk) {
        hi = mid;
      } else {
        lo = mid;
      }
    }
    const uint32_t dstar = static_cast<uint32_t>(hi);
    // ---- eligible candidates (distance <= d*, finite), compacted into the histogram area
    uint32_t n_elig = 0;
#pragma unroll
    for (int m = 0; m < kListCap / 32; ++m) {
      const bool ok = dist[m] <= dstar && M - dist[m] != kKeyNegInf;
      const unsigned b = __ballot_sync(0xffffffffu, ok);
      if (ok) elig[n_elig + __popc(b & ((1u << lane) - 1u))] = tokn[m];
      n_elig += __popc(b);
    }
    __syncwarp();
    score_list(elig, n_elig, vals, seed32, off64, prm.temperature, best);
  } else {
    // exact binary search over keys: count(value >= lo) >= k > count(value >= hi)
    uint32_t lo = kKeyNegInf, hi = M + 1;
    while (hi - lo > 1) {
      const uint32_t mid = (lo + hi) >> 1;
      if (count_ge(vals, key_value(mid)) >= kk) {
        lo = mid;
      } else {
        hi = mid;
      }
    }
#pragma unroll 1
    for (int i = 0; i < 8; ++i) {
      const int ch = lane + 32 * i;
      if (ch < kVocabChunks) {
        for (int e = 0; e < 8; ++e) {
          const int t = 8 * ch + e;
          const uint32_t key = sample_key(vals[t]);
          if (key >= lo && key != kKeyNegInf) {
            const float g = clamped_gumbel(philox_uniform(seed32, off64 + static_cast<uint64_t>(t)));
            keep_best(best, __fadd_rn(__fdiv_rn(bits2f(vals[t]), prm.temperature), g), t);
          }
        }
      }
    }
  }
  best = warp_best(best);
  int token = best.id;
  if (token >= kVocab || best.score == -CUDART_INF_F) {
    invalid = 1;
    token = 0;
  }
  *invalid_out = invalid;
  return token;
}


// ---------------------------------------------------------------------------
// Group sampler: W warps (32 W threads, named barrier `bar_id`) sample one
// session row together.  Same contract and the same result as sample_row;
// the row maximum M (order key) comes from the head epilogue.  The row is
// split into W ranges of 8-value chunks; window counts, the candidate list,
// the distance histogram that gives the exact k-th largest, and the scoring
// of the eligible tokens are shared across the group.  Eligible tokens are
// ranked with the fast Gumbel and those within kVerifyMargin of the best are
// rescored with the contract's correctly rounded one (as score_list does).
// ---------------------------------------------------------------------------

struct GroupScratch {
  uint32_t cnt[8][4];   // per-warp window counts
  uint32_t cnt2[8][2];  // per-warp counts of the whole-row search (alternating)
  uint32_t hist[256];   // candidates per distance below the maximum
  float best_score[8];
  int32_t best_id[8];
};

__device__ __forceinline__ void group_bar(int bar_id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(threads) : "memory");
}

template <int W>
__device__ int sample_group(const RowSample& rs, uint32_t M, const SamplingParams& prm, uint32_t* list32,
                            GroupScratch& gs, int bar_id, int* invalid_out) {
  constexpr int kThreadsG = 32 * W;
  constexpr int kCpw = (kVocabChunks + W - 1) / W;  // chunks per warp
  constexpr int kIt = (kCpw + 31) / 32;             // chunks per lane
  const int lane = threadIdx.x & 31;
  const int g = (threadIdx.x >> 5) % W;
  const int tid = 32 * g + lane;
  const int ch0 = kCpw * g;
  const int ch1 = ch0 + kCpw < kVocabChunks ? ch0 + kCpw : kVocabChunks;
  const bool unfinished = rs.flags & 1u, finished = rs.flags & 2u, forbid = rs.flags & 4u;
  const uint16_t* vals = rs.vals;
  if (prm.argmax) {
    *invalid_out = (rs.nonfinite || M == kKeyNegInf) ? 1 : 0;
    if (M == kKeyNegInf) return 0;
    int first = kVocab;
#pragma unroll
    for (int i = kIt - 1; i >= 0; --i) {
      const int ch = ch0 + lane + 32 * i;
      if (ch < ch1) {
        const uint4 q = *reinterpret_cast<const uint4*>(vals + 8 * ch);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 3; e >= 0; --e) {
          if (sample_key(w[e] >> 16) == M) first = 8 * ch + 2 * e + 1;
          if (sample_key(w[e] & 0xffffu) == M) first = 8 * ch + 2 * e;
        }
      }
    }
    first = static_cast<int>(__reduce_min_sync(0xffffffffu, static_cast<uint32_t>(first)));
    if (lane == 0) gs.best_id[g] = first;
    group_bar(bar_id, kThreadsG);
    int t = kVocab;
#pragma unroll
    for (int j = 0; j < W; ++j) t = gs.best_id[j] < t ? gs.best_id[j] : t;
    return t;
  }
  int invalid = (rs.nonfinite || (unfinished && finished) || (finished && forbid)) ? 1 : 0;
  const int64_t seed = rs.seed, counter = rs.counter;
  const bool seed_valid = seed >= 0 && static_cast<uint64_t>(seed) < (1ull << 32);
  const bool counter_valid = counter >= 0 && counter <= kMaxCounter;
  if (!seed_valid || !counter_valid) invalid = 1;
  if (finished) {  // only EOS (value 0) is finite: it is the only eligible token
    *invalid_out = invalid;
    return kEosId;
  }
  if (M == kKeyNegInf) {
    *invalid_out = 1;
    return 0;
  }
  const uint32_t seed32 = seed_valid ? static_cast<uint32_t>(seed) : 0u;
  const uint64_t off64 = counter_valid ? static_cast<uint64_t>(counter) * kPhiloxStride : 0ull;
  const uint32_t kk = static_cast<uint32_t>(prm.top_k);

  // ---- window counts: values within 32 / 64 / 128 / 256 key steps of the maximum
  __nv_bfloat162 lim[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) lim[j] = __bfloat162bfloat162(key_value(M + 1 < (32u << j) ? 0u : M + 1 - (32u << j)));
  __nv_bfloat162 acc[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) acc[j] = __float2bfloat162_rn(0.f);
#pragma unroll
  for (int i = 0; i < kIt; ++i) {
    const int ch = ch0 + lane + 32 * i;
    if (ch < ch1) {
      const uint4 q = *reinterpret_cast<const uint4*>(vals + 8 * ch);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int e = 0; e < 4; ++e)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[j] = __hadd2(acc[j], __hge2(bf2_of(w[e]), lim[j]));
    }
  }
  uint32_t mine4[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f2 = __bfloat1622float2(acc[j]);
    mine4[j] = static_cast<uint32_t>(f2.x + f2.y);
    const uint32_t wt = __reduce_add_sync(0xffffffffu, mine4[j]);
    if (lane == 0) gs.cnt[g][j] = wt;
  }
  for (int i = tid; i < 256; i += kThreadsG) gs.hist[i] = 0;
  group_bar(bar_id, kThreadsG);
  uint32_t tot[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    tot[j] = 0;
#pragma unroll
    for (int q = 0; q < W; ++q) tot[j] += gs.cnt[q][j];
  }
  int win = 4;
#pragma unroll
  for (int j = 3; j >= 0; --j) win = tot[j] >= kk ? j : win;

  Best best{-CUDART_INF_F, kVocab};
  if (win < 4 && tot[win] <= static_cast<uint32_t>(kListCap)) {
    const __nv_bfloat162 limw = win == 0 ? lim[0] : (win == 1 ? lim[1] : (win == 2 ? lim[2] : lim[3]));
    const uint32_t mine = win == 0 ? mine4[0] : (win == 1 ? mine4[1] : (win == 2 ? mine4[2] : mine4[3]));
    const uint32_t n_cand = tot[win];
    uint32_t pos = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, pos, o);
      if (lane >= o) pos += y;
    }
    pos -= mine;
#pragma unroll
    for (int q = 0; q < W; ++q) pos += q < g ? gs.cnt[q][win] : 0u;
    // ---- the window's tokens, with their keys
#pragma unroll
    for (int i = 0; i < kIt; ++i) {
      const int ch = ch0 + lane + 32 * i;
      if (ch < ch1) {
        const uint4 q = *reinterpret_cast<const uint4*>(vals + 8 * ch);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t m = __hge2_mask(bf2_of(w[e]), limw);
          if (m & 1u) list32[pos++] = (sample_key(w[e] & 0xffffu) << 16) | static_cast<uint32_t>(8 * ch + 2 * e);
          if (m >> 31) list32[pos++] = (sample_key(w[e] >> 16) << 16) | static_cast<uint32_t>(8 * ch + 2 * e + 1);
        }
      }
    }
    group_bar(bar_id, kThreadsG);
    for (uint32_t e = tid; e < n_cand; e += kThreadsG) atomicAdd(&gs.hist[M - (list32[e] >> 16)], 1u);
    group_bar(bar_id, kThreadsG);
    // smallest d with (candidates at distance <= d) >= k: lane holds bins [8 lane, +8)
    uint32_t h[8], part = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      h[j] = gs.hist[8 * lane + j];
      part += h[j];
    }
    uint32_t incl = part;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const unsigned reach = __ballot_sync(0xffffffffu, incl >= kk);
    const int L = __ffs(reach) - 1;  // tot[win] >= k, so some lane reaches k
    uint32_t dstar = 0;
    if (lane == L) {
      uint32_t c = incl - part;  // candidates in the bins below this lane's
      bool found = false;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c += h[j];
        if (!found && c >= kk) {
          dstar = 8 * L + j;
          found = true;
        }
      }
    }
    dstar = __shfl_sync(0xffffffffu, dstar, L);
    // ---- eligible candidates (distance <= d*, finite): fast scores, the
    // group's best fast score, then the exact score only for candidates
    // within kVerifyMargin of it (a lone one is the winner as it stands)
    constexpr int kPer = kListCap / kThreadsG;
    float fs[kPer];
    int tk[kPer];
    float bf = -CUDART_INF_F;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      fs[i] = -CUDART_INF_F;
      tk[i] = kVocab;
      const uint32_t e = tid + kThreadsG * i;
      if (e < n_cand) {
        const uint32_t v = list32[e];
        const uint32_t key = v >> 16;
        if (M - key <= dstar && key != kKeyNegInf) {
          const int t = static_cast<int>(v & 0xffffu);
          tk[i] = t;
          fs[i] = __fadd_rn(__fdiv_rn(bits2f(vals[t]), prm.temperature),
                            fast_gumbel(philox_uniform(seed32, off64 + static_cast<uint64_t>(t))));
          bf = fmaxf(bf, fs[i]);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) bf = fmaxf(bf, __shfl_xor_sync(0xffffffffu, bf, o));
    if (lane == 0) gs.best_score[g] = bf;
    group_bar(bar_id, kThreadsG);
    float gbf = -CUDART_INF_F;
#pragma unroll
    for (int q = 0; q < W; ++q) gbf = fmaxf(gbf, gs.best_score[q]);
    const float cut = gbf - kVerifyMargin;
    uint32_t near = 0;
#pragma unroll
    for (int i = 0; i < kPer; ++i) near += (tk[i] < kVocab && fs[i] >= cut) ? 1u : 0u;
    near = __reduce_add_sync(0xffffffffu, near);
    if (lane == 0) gs.cnt2[g][0] = near;
    group_bar(bar_id, kThreadsG);
    uint32_t tot_near = 0;
#pragma unroll
    for (int q = 0; q < W; ++q) tot_near += gs.cnt2[q][0];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      if (tk[i] < kVocab && fs[i] >= cut) {
        keep_best(best,
                  tot_near == 1 ? fs[i]
                                : exact_score(bits2f(vals[tk[i]]), prm.temperature, seed32,
                                              off64 + static_cast<uint64_t>(tk[i])),
                  tk[i]);
      }
    }
  } else {
    // exact search over keys: count(value >= lo) >= k > count(value >= hi)
    uint32_t lo = kKeyNegInf, hi = M + 1;
    int it = 0;
    while (hi - lo > 1) {
      const uint32_t mid = (lo + hi) >> 1;
      const __nv_bfloat162 t2 = __bfloat162bfloat162(key_value(mid));
      __nv_bfloat162 a2 = __float2bfloat162_rn(0.f);
#pragma unroll
      for (int i = 0; i < kIt; ++i) {
        const int ch = ch0 + lane + 32 * i;
        if (ch < ch1) {
          const uint4 q = *reinterpret_cast<const uint4*>(vals + 8 * ch);
          a2 = __hadd2(a2, __hge2(bf2_of(q.x), t2));
          a2 = __hadd2(a2, __hge2(bf2_of(q.y), t2));
          a2 = __hadd2(a2, __hge2(bf2_of(q.z), t2));
          a2 = __hadd2(a2, __hge2(bf2_of(q.w), t2));
        }
      }
      const float2 f2 = __bfloat1622float2(a2);
      const uint32_t wt = __reduce_add_sync(0xffffffffu, static_cast<uint32_t>(f2.x + f2.y));
      if (lane == 0) gs.cnt2[g][it & 1] = wt;
      group_bar(bar_id, kThreadsG);
      uint32_t c = 0;
#pragma unroll
      for (int q = 0; q < W; ++q) c += gs.cnt2[q][it & 1];
      if (c >= kk) {
        lo = mid;
      } else {
        hi = mid;
      }
      ++it;
    }
#pragma unroll 1
    for (int i = 0; i < kIt; ++i) {
      const int ch = ch0 + lane + 32 * i;
      if (ch < ch1) {
        for (int e = 0; e < 8; ++e) {
          const int t = 8 * ch + e;
          const uint32_t key = sample_key(vals[t]);
          if (key >= lo && key != kKeyNegInf) {
            keep_best(best, exact_score(bits2f(vals[t]), prm.temperature, seed32, off64 + static_cast<uint64_t>(t)), t);
          }
        }
      }
    }
  }
  best = warp_best(best);
  if (lane == 0) {
    gs.best_score[g] = best.score;
    gs.best_id[g] = best.id;
  }
  group_bar(bar_id, kThreadsG);
  Best all{-CUDART_INF_F, kVocab};
#pragma unroll
  for (int q = 0; q < W; ++q) keep_best(all, gs.best_score[q], gs.best_id[q]);
  int token = all.id;
  if (token >= kVocab || all.score == -CUDART_INF_F) {
    invalid = 1;
    token = 0;
  }
  *invalid_out = invalid;
  return token;
}

}  // namespace
}  // namespace mtt
