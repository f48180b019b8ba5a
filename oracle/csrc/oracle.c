/*
 * CPU oracle for the MagpieTTS-RT per-frame Local AR sampling path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
 * calls this file; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg use it, and only as the checker.
 *
 * Every function restates the reference's arithmetic in plain C and cites the
 * reference file:line it follows (paths relative to the reference project):
 *
 *   plugins/local_ar_plugins.cu:1149-1370   philox_word / philox_uniform /
 *                                            guided_logit / clamped_gumbel /
 *                                            sampling_kernel
 *   plugins/local_ar_plugins.cu:1372-1495   eos_projection / eos_reduce /
 *                                            eos_finalize
 *   tools/export/local_ar_wrapper.py:153-286 philox_uniform, _reference_sample
 *   tools/export/local_ar_wrapper.py:424-476 _reference_eos
 *   reference/nemo-oracle-overlay/.../magpietts_fused_sampling.py:42-197
 *                                            constrained logits, argmax mode
 *   tools/export/main_decoder_wrapper.py:796-810, magpietts.py:1973-1985
 *                                            next-frame embedding sum
 *   src/runtime/synthesis_kernels.cu:53-86   finalize_local_step
 *
 * Build with -ffp-contract=off: every float/double operation must round
 * exactly once, in program order, so that the CUDA kernels (which use the
 * explicit _rn intrinsics for the same operations) produce identical bits.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define ORC_VOCAB 2024
#define ORC_CODEBOOK 2016
#define ORC_EOS 2017
#define ORC_COMPACT_EOS_VOCAB 2017
#define ORC_EMBED 768
#define ORC_POSITIONS 16
#define ORC_CODEBOOKS 8
#define ORC_FRAMES 2
#define ORC_PHILOX_STRIDE 2048
/* (INT64_MAX - (2048 - 1)) / 2048, plugins/local_ar_plugins.cu:45-47 */
#define ORC_MAX_COUNTER ((int64_t)((INT64_MAX - (ORC_PHILOX_STRIDE - 1)) / ORC_PHILOX_STRIDE))

/* ------------------------------------------------------------------------ */
/* bf16 <-> f32                                                              */
/* ------------------------------------------------------------------------ */

static inline float bits_to_f32(uint32_t u) {
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

static inline uint32_t f32_to_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof u);
  return u;
}

float orc_bf16_to_f32(uint16_t h) { return bits_to_f32((uint32_t)h << 16); }

/* Round-to-nearest-even f32 -> bf16; NaN stays NaN (quiet). */
uint16_t orc_f32_to_bf16(float f) {
  uint32_t u = f32_to_bits(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) {
    return (uint16_t)((u >> 16) | 0x0040u);
  }
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float round_bf16(float f) { return orc_bf16_to_f32(orc_f32_to_bf16(f)); }

/* ------------------------------------------------------------------------ */
/* Philox-4x32-10, only word c0 used.                                        */
/* plugins/local_ar_plugins.cu:1149-1169, local_ar_wrapper.py:153-175        */
/* ------------------------------------------------------------------------ */

uint32_t orc_philox_word(uint32_t seed, uint64_t offset) {
  uint32_t c0 = (uint32_t)offset, c1 = (uint32_t)(offset >> 32), c2 = 0, c3 = 0;
  uint32_t k0 = seed, k1 = 0;
  for (int round = 0; round < 10; ++round) {
    const uint32_t p0 = c0, p2 = c2;
    c0 = (uint32_t)(((uint64_t)0xCD9E8D57u * p2) >> 32) ^ c1 ^ k0;
    c2 = (uint32_t)(((uint64_t)0xD2511F53u * p0) >> 32) ^ c3 ^ k1;
    c1 = 0xCD9E8D57u * p2;
    c3 = 0xD2511F53u * p0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c0;
}

/* signed-magnitude(c0) * 4.6566127342e-10f (local_ar_plugins.cu:1171-1180). */
float orc_philox_uniform(uint32_t seed, uint64_t offset) {
  const int32_t w = (int32_t)orc_philox_word(seed, offset);
  const int64_t magnitude = w < 0 ? -(int64_t)w - 1 : (int64_t)w;
  return (float)magnitude * 4.6566127342e-10f;
}

/* ------------------------------------------------------------------------ */
/* Natural log, correctly rounded to f32 for the Gumbel domain.              */
/*                                                                           */
/* The reference's three implementations of -log(-log u) each round their   */
/* own f32 log (CUDA __logf, Triton tl.log, PyTorch CPU log); none is        */
/* correctly rounded.  This build fixes the rounding: each log is evaluated */
/* in double by a table-driven reduction (Tang's method) and rounded once   */
/* to f32.  x = 2^e * m with m in [sqrt(1/2), sqrt(2)); j = nearest(64(m-1)) */
/* picks c_j = 1 + j/64 with a 29-bit inv_j ~ 1/c_j (so m * inv_j is exact) */
/* and L_j = -log(inv_j); t = m * inv_j - 1 (|t| < 0.0113, exact);          */
/* log(m) = L_j + log1p(t), log1p(t) = t + t^2 q(t) with 10 series terms.   */
/* j = 0 has c = 1 exactly, so results near log 1 = 0 do not cancel.        */
/* The CUDA kernels run the identical sequence of IEEE double operations    */
/* (explicit fma / mul / add), so the two agree bit for bit by construction.*/
/* Valid for positive normal f32 inputs.                                    */
/* ------------------------------------------------------------------------ */

static const double kLn2Hi = 0x1.62e42feep-1;
static const double kLn2Lo = 1.9082149292705877e-10;
static const double kSqrt2 = 1.4142135623730951;

/* {inv_j, L_j} for j = -19 .. 27 */
static const double kLogTable[47][2] = {
    {0x1.6c16c17000000p+0, -0x1.68ac83f4c6a14p-2},  /* j = -19 */
    {0x1.642c859000000p+0, -0x1.522ae0718a3d8p-2},  /* j = -18 */
    {0x1.5c9882c000000p+0, -0x1.3c25278733184p-2},  /* j = -17 */
    {0x1.5555555000000p+0, -0x1.269621034db92p-2},  /* j = -16 */
    {0x1.4e5e0a7000000p+0, -0x1.1178e8197e47cp-2},  /* j = -15 */
    {0x1.47ae148000000p+0, -0x1.f991c6eb3b379p-3},  /* j = -14 */
    {0x1.4141414000000p+0, -0x1.d1037f1e55e7bp-3},  /* j = -13 */
    {0x1.3b13b14000000p+0, -0x1.a93ed3e8ad9e3p-3},  /* j = -12 */
    {0x1.3521cfb000000p+0, -0x1.823c16431a3c2p-3},  /* j = -11 */
    {0x1.2f684be000000p+0, -0x1.5bf406dd43db2p-3},  /* j = -10 */
    {0x1.29e412a000000p+0, -0x1.365fcb0d59016p-3},  /* j = -9 */
    {0x1.2492492000000p+0, -0x1.1178e8027e47cp-3},  /* j = -8 */
    {0x1.1f7047e000000p+0, -0x1.da727670446a2p-4},  /* j = -7 */
    {0x1.1a7b961000000p+0, -0x1.9335e5bd94989p-4},  /* j = -6 */
    {0x1.15b1e5f000000p+0, -0x1.4d31156607eacp-4},  /* j = -5 */
    {0x1.1111111000000p+0, -0x1.08598b49e3a07p-4},  /* j = -4 */
    {0x1.0c97150000000p+0, -0x1.894aa1c9fb343p-5},  /* j = -3 */
    {0x1.0842108000000p+0, -0x1.0415d81e74444p-5},  /* j = -2 */
    {0x1.0410410000000p+0, -0x1.0205648935847p-6},  /* j = -1 */
    {0x1.0000000000000p+0, 0x0.0p+0},  /* j = 0 */
    {0x1.f81f820000000p-1, 0x1.fc0a890fc03e4p-7},  /* j = 1 */
    {0x1.f07c1f0000000p-1, 0x1.f829b1e783300p-6},  /* j = 2 */
    {0x1.e9131ac000000p-1, 0x1.77458f532dcfcp-5},  /* j = 3 */
    {0x1.e1e1e1e000000p-1, 0x1.f0a30c21162a6p-5},  /* j = 4 */
    {0x1.dae6077000000p-1, 0x1.341d793bbd1d1p-4},  /* j = 5 */
    {0x1.d41d41d000000p-1, 0x1.6f0d28d256b4cp-4},  /* j = 6 */
    {0x1.cd85689000000p-1, 0x1.a926d3a6ad563p-4},  /* j = 7 */
    {0x1.c71c71c000000p-1, 0x1.e2707722af2e6p-4},  /* j = 8 */
    {0x1.c0e0704000000p-1, 0x1.0d77e7a908e59p-3},  /* j = 9 */
    {0x1.bacf915000000p-1, 0x1.29552f6fff523p-3},  /* j = 10 */
    {0x1.b4e81b5000000p-1, 0x1.44d2b6c5b7d1ep-3},  /* j = 11 */
    {0x1.af286bd000000p-1, 0x1.5ff306ee793d4p-3},  /* j = 12 */
    {0x1.a98ef60000000p-1, 0x1.7ab890410d909p-3},  /* j = 13 */
    {0x1.a41a41a000000p-1, 0x1.9525a9e3456b4p-3},  /* j = 14 */
    {0x1.9ec8e95000000p-1, 0x1.af3c94ed0bff3p-3},  /* j = 15 */
    {0x1.999999a000000p-1, 0x1.c8ff7c59a9a22p-3},  /* j = 16 */
    {0x1.948b0fd000000p-1, 0x1.e27076d5af2e6p-3},  /* j = 17 */
    {0x1.8f9c190000000p-1, 0x1.fb9186b5e3e2bp-3},  /* j = 18 */
    {0x1.8acb90f000000p-1, 0x1.0a324e38b90e3p-2},  /* j = 19 */
    {0x1.8618618000000p-1, 0x1.1675cacaba60ep-2},  /* j = 20 */
    {0x1.8181818000000p-1, 0x1.22941fc0f7966p-2},  /* j = 21 */
    {0x1.7d05f41000000p-1, 0x1.2e8e2bc311d31p-2},  /* j = 22 */
    {0x1.78a4c81000000p-1, 0x1.3a64c56b145eap-2},  /* j = 23 */
    {0x1.745d174000000p-1, 0x1.4618bc31c5ec2p-2},  /* j = 24 */
    {0x1.702e05c000000p-1, 0x1.51aad874df82dp-2},  /* j = 25 */
    {0x1.6c16c17000000p-1, 0x1.5d1bdbea809cap-2},  /* j = 26 */
    {0x1.6816817000000p-1, 0x1.686c81d3314afp-2},  /* j = 27 */
};

double orc_log_double(float x) {
  const uint32_t bits = f32_to_bits(x);
  int exponent = (int)((bits >> 23) & 0xffu) - 127;
  double m = (double)bits_to_f32((bits & 0x007fffffu) | 0x3f800000u); /* [1,2) */
  if (m > kSqrt2) {
    m = m * 0.5;
    exponent += 1;
  }
  const int j = (int)lrint((m - 1.0) * 64.0);
  const double inv = kLogTable[j + 19][0];
  const double L = kLogTable[j + 19][1];
  const double t = fma(m, inv, -1.0);
  double q = 0x1.745d1745d1746p-4;
  q = fma(q, t, -0x1.999999999999ap-4);
  q = fma(q, t, 0x1.c71c71c71c71cp-4);
  q = fma(q, t, -0x1.0000000000000p-3);
  q = fma(q, t, 0x1.2492492492492p-3);
  q = fma(q, t, -0x1.5555555555555p-3);
  q = fma(q, t, 0x1.999999999999ap-3);
  q = fma(q, t, -0x1.0000000000000p-2);
  q = fma(q, t, 0x1.5555555555555p-2);
  q = fma(q, t, -0x1.0000000000000p-1);
  const double t2 = t * t;
  const double log_m = L + fma(t2, q, t);
  const double e = (double)exponent;
  return e * kLn2Hi + (e * kLn2Lo + log_m);
}

float orc_log_f32(float x) { return (float)orc_log_double(x); }

/* clamp then -log(-log u), two f32-rounded logs (local_ar_plugins.cu:1193-1196,
 * local_ar_wrapper.py:260-261). */
float orc_clamped_gumbel(float u) {
  u = fmaxf(0.00000006f, fminf(0.99999994f, u));
  const float inner = orc_log_f32(u);
  return -orc_log_f32(-inner);
}

/* ------------------------------------------------------------------------ */
/* CFG: bf16(bf16(cond * scale) + uncond * (1 - scale))                       */
/* local_ar_plugins.cu:1182-1191, magpietts_fused_sampling.py:69-72           */
/* ------------------------------------------------------------------------ */

float orc_guided_logit(uint16_t cond, uint16_t uncond, float cfg_scale) {
  const float scaled = round_bf16(orc_bf16_to_f32(cond) * cfg_scale);
  const float sum = scaled + orc_bf16_to_f32(uncond) * (1.0f - cfg_scale);
  return round_bf16(sum);
}

/* ------------------------------------------------------------------------ */
/* One sampling call.                                                         */
/* ------------------------------------------------------------------------ */

enum {
  ORC_LOGITS_BF16_CFG = 0, /* logits = [2][V] bf16: cond row, uncond row */
  ORC_LOGITS_BF16 = 1,     /* logits = [V] bf16, no CFG */
  ORC_LOGITS_F32 = 2       /* logits = [V] f32, no CFG */
};

typedef struct {
  int32_t top_k;
  float temperature;
  float cfg_scale;
  int32_t argmax; /* 1: greedy mode (magpietts_fused_sampling.py:136-197) */
} orc_sampling_params;

static void constrained_values(const void* logits, int logits_kind, int unfinished,
                               int finished, int forbid_eos, float cfg_scale,
                               float* values, int* nonfinite_out) {
  int nonfinite = 0;
  for (int t = 0; t < ORC_VOCAB; ++t) {
    float v;
    if (logits_kind == ORC_LOGITS_BF16_CFG) {
      const uint16_t* l = (const uint16_t*)logits;
      v = orc_guided_logit(l[t], l[ORC_VOCAB + t], cfg_scale);
    } else if (logits_kind == ORC_LOGITS_BF16) {
      v = orc_bf16_to_f32(((const uint16_t*)logits)[t]);
    } else {
      v = ((const float*)logits)[t];
    }
    if (!isfinite(v)) {
      nonfinite = 1;
      v = -INFINITY;
    }
    const int forbidden_special = t >= ORC_CODEBOOK && t != ORC_EOS;
    if (forbidden_special || ((unfinished || forbid_eos) && t == ORC_EOS)) {
      v = -INFINITY;
    }
    if (finished) {
      v = t == ORC_EOS ? 0.0f : -INFINITY;
    }
    values[t] = v;
  }
  *nonfinite_out = nonfinite;
}

/* k-th largest (1-based), inclusive threshold of torch.topk(...).values[-1]. */
static float kth_largest(const float* values, int k) {
  /* counting select over the order-preserving u32 image of the floats */
  uint32_t keys[ORC_VOCAB];
  for (int t = 0; t < ORC_VOCAB; ++t) {
    uint32_t u = f32_to_bits(values[t]);
    keys[t] = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  }
  uint32_t prefix = 0, mask = 0;
  int remaining = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    int hist[256] = {0};
    for (int t = 0; t < ORC_VOCAB; ++t) {
      if ((keys[t] & mask) == prefix) hist[(keys[t] >> shift) & 0xffu]++;
    }
    int digit = 255;
    for (; digit > 0; --digit) {
      if (hist[digit] >= remaining) break;
      remaining -= hist[digit];
    }
    prefix |= (uint32_t)digit << shift;
    mask |= 0xffu << shift;
  }
  const uint32_t key = prefix;
  const uint32_t u = (key & 0x80000000u) ? (key & 0x7fffffffu) : ~key;
  return bits_to_f32(u);
}

/*
 * Sample one (stream, position).  Follows sampling_kernel
 * (local_ar_plugins.cu:1211-1370) for top-k mode and
 * _fused_argmax_embedding_kernel (magpietts_fused_sampling.py:136-197) for
 * argmax mode.  Returns the chosen token; writes the updated counter and the
 * invalid flag.
 */
int64_t orc_sample(const void* logits, int logits_kind, int unfinished, int finished,
                   int forbid_eos, int64_t seed, int64_t counter,
                   const orc_sampling_params* params, int64_t* counter_out,
                   int32_t* invalid_out) {
  float values[ORC_VOCAB];
  int nonfinite = 0;
  constrained_values(logits, logits_kind, unfinished, finished, forbid_eos,
                     params->cfg_scale, values, &nonfinite);
  int invalid = nonfinite;
  int finite_candidates = 0;
  for (int t = 0; t < ORC_VOCAB; ++t) finite_candidates += isfinite(values[t]) ? 1 : 0;
  if (finite_candidates == 0) invalid = 1;

  if (params->argmax) {
    int best = 0;
    for (int t = 1; t < ORC_VOCAB; ++t) {
      if (values[t] > values[best]) best = t;
    }
    *counter_out = counter;
    *invalid_out = invalid;
    return best;
  }

  if (unfinished && finished) invalid = 1;
  if (finished && forbid_eos) invalid = 1;
  const int seed_valid = seed >= 0 && (uint64_t)seed < ((uint64_t)1 << 32);
  const int counter_valid = counter >= 0 && counter <= ORC_MAX_COUNTER;
  if (!seed_valid || !counter_valid) invalid = 1;

  const float threshold = kth_largest(values, params->top_k);
  const uint32_t seed32 = seed_valid ? (uint32_t)seed : 0u;
  const uint64_t base = counter_valid ? (uint64_t)counter * ORC_PHILOX_STRIDE : 0u;
  float best_score = -INFINITY;
  int best_id = ORC_VOCAB;
  for (int t = 0; t < ORC_VOCAB; ++t) {
    if (values[t] < threshold) continue;
    const float g = orc_clamped_gumbel(orc_philox_uniform(seed32, base + (uint64_t)t));
    const float score = values[t] / params->temperature + g;
    if (score > best_score || (score == best_score && t < best_id)) {
      best_score = score;
      best_id = t;
    }
  }
  if (best_id >= ORC_VOCAB || best_score == -INFINITY) {
    invalid = 1;
    best_id = 0;
  }
  *counter_out = counter_valid ? counter + 1 : counter;
  *invalid_out = invalid;
  return best_id;
}

/* Batched convenience: n independent calls, row stride in logits elements. */
void orc_sample_batch(const void* logits, int logits_kind, int64_t row_stride, int n,
                      const uint8_t* unfinished, const uint8_t* finished,
                      const uint8_t* forbid_eos, const int64_t* seed,
                      const int64_t* counter, const orc_sampling_params* params,
                      int64_t* token, int64_t* counter_out, int32_t* invalid) {
  const size_t esize = logits_kind == ORC_LOGITS_F32 ? 4 : 2;
  for (int i = 0; i < n; ++i) {
    const char* row = (const char*)logits + (size_t)i * (size_t)row_stride * esize;
    token[i] = orc_sample(row, logits_kind, unfinished[i], finished[i], forbid_eos[i],
                          seed[i], counter[i], params, &counter_out[i], &invalid[i]);
  }
}

/* ------------------------------------------------------------------------ */
/* EOS                                                                       */
/* ------------------------------------------------------------------------ */

/*
 * Guided EOS logits for the 16 x 2017 compact rows (2016 codes + EOS) of the
 * Main Decoder final projection (eos_projection_kernel,
 * local_ar_plugins.cu:1372-1432).  Dot products are taken in double and
 * rounded once to f32 (the CUDA kernel accumulates in f32; the two agree to
 * within f32 accumulation error, which the tests bound).
 */
void orc_eos_guided(const uint16_t* hidden /*[2][768]*/, const uint16_t* weight /*[16*2024][768]*/,
                    const uint16_t* bias /*[16*2024]*/, float cfg_scale,
                    float* guided /*[16][2017]*/) {
  for (int p = 0; p < ORC_POSITIONS; ++p) {
    for (int ct = 0; ct < ORC_COMPACT_EOS_VOCAB; ++ct) {
      const int token = ct == ORC_CODEBOOK ? ORC_EOS : ct;
      const size_t row = (size_t)p * ORC_VOCAB + (size_t)token;
      double dc = 0.0, du = 0.0;
      for (int k = 0; k < ORC_EMBED; ++k) {
        const double w = orc_bf16_to_f32(weight[row * ORC_EMBED + k]);
        dc += (double)orc_bf16_to_f32(hidden[k]) * w;
        du += (double)orc_bf16_to_f32(hidden[ORC_EMBED + k]) * w;
      }
      const float b = orc_bf16_to_f32(bias[row]);
      const float c = round_bf16((float)dc + b);
      const float u = round_bf16((float)du + b);
      const float u_scaled = round_bf16(u * (1.0f - cfg_scale));
      guided[p * ORC_COMPACT_EOS_VOCAB + ct] = round_bf16(u_scaled + c * cfg_scale);
    }
  }
}

/*
 * eos_reduce_kernel + eos_finalize_kernel (local_ar_plugins.cu:1434-1495):
 * per position EOS if the EOS logit beats every code logit or the sampled
 * token is EOS; any over codebooks; first frame wins.  guided may be NULL when
 * EOS evaluation is skipped (unfinished || forbid_eos || finished).
 */
int32_t orc_eos_end_frame(const float* guided, const int64_t* codec_tokens /*[8][2]*/,
                          int unfinished, int finished, int forbid_eos) {
  int frame_eos[ORC_FRAMES] = {0, 0};
  for (int p = 0; p < ORC_POSITIONS; ++p) {
    const int frame = p / ORC_CODEBOOKS;
    if (finished) {
      frame_eos[frame] = 1;
      continue;
    }
    if (unfinished || forbid_eos) continue;
    float best = -INFINITY;
    for (int t = 0; t < ORC_CODEBOOK; ++t) best = fmaxf(best, guided[p * ORC_COMPACT_EOS_VOCAB + t]);
    const float eos_logit = guided[p * ORC_COMPACT_EOS_VOCAB + ORC_CODEBOOK];
    const int codebook = p % ORC_CODEBOOKS;
    const int sampled = codec_tokens[codebook * ORC_FRAMES + frame] == ORC_EOS;
    if (eos_logit > best || sampled) frame_eos[frame] = 1;
  }
  return frame_eos[0] ? 0 : (frame_eos[1] ? 1 : -1);
}

/* ------------------------------------------------------------------------ */
/* Next-frame embedding: sum_{p=0..15} table_p[token_p], each add rounded to  */
/* bf16, then / 16 (main_decoder_wrapper.py:796-810; magpietts.py:1973-1985). */
/* ------------------------------------------------------------------------ */

void orc_embedding_sum(const uint16_t* tables /*[16][2024][768]*/, const int64_t* tokens /*[16]*/,
                       uint16_t* out /*[768]*/) {
  for (int k = 0; k < ORC_EMBED; ++k) {
    float acc = 0.0f;
    for (int p = 0; p < ORC_POSITIONS; ++p) {
      const int64_t tok = tokens[p];
      const float v = orc_bf16_to_f32(tables[((size_t)p * ORC_VOCAB + (size_t)tok) * ORC_EMBED + k]);
      acc = p == 0 ? v : round_bf16(acc + v);
    }
    out[k] = orc_f32_to_bf16(acc / 16.0f);
  }
}

/* Position-major tokens [16] -> codec_tokens [8][2] with p = frame*8 + codebook
 * (local_ar_wrapper.py:736-741). */
void orc_codec_layout(const int64_t* position_major, int64_t* codec_tokens) {
  for (int p = 0; p < ORC_POSITIONS; ++p) {
    const int frame = p / ORC_CODEBOOKS, codebook = p % ORC_CODEBOOKS;
    codec_tokens[codebook * ORC_FRAMES + frame] = position_major[p];
  }
}

/* finalize_local_step_kernel (src/runtime/synthesis_kernels.cu:53-86). */
void orc_finalize_local_step(const int64_t* step_codec_tokens /*[16]*/, int64_t* aggregate /*[8][8]*/,
                             uint32_t frame_offset, int32_t invalid_rows, int32_t end_frame_index,
                             int32_t* step_invalid, int32_t* step_end, int64_t updated_counter,
                             int64_t* counter, uint8_t* generation_finished) {
  for (int i = 0; i < ORC_CODEBOOKS * ORC_FRAMES; ++i) {
    const int codebook = i / ORC_FRAMES, frame = i % ORC_FRAMES;
    aggregate[codebook * 8 + (int)frame_offset + frame] = step_codec_tokens[i];
  }
  *step_invalid = invalid_rows;
  *step_end = end_frame_index;
  *counter = updated_counter;
  if (end_frame_index == 0 || end_frame_index == 1) *generation_finished = 1;
}
