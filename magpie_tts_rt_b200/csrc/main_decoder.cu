// Main Decoder one-step for N sessions (both CFG rows each) per launch
// sequence: the decoder position that produces the Local AR's input hidden
// state and the alignment controller's scores.
//
// Reference: tools/export/main_decoder_wrapper.py:778-911
// (MainDecoderStepWrapper.forward: one TensorRT engine per session per step,
// K/V state as explicit engine I/O, src/runtime/synthesis_pipeline.cpp:
// 572-648).  Per layer:
//   add_ln     x = bf16(x + o); LN(x) (fused; the layer-0 form adds the
//              position embedding to the codec embedding sum)
//   GEMM       q|k|v = LN(x) W_qkv^T                  (tcgen05, bf16 in/out, f32 accumulate)
//   self_attn  k, v written at the session's position; attention of the 12
//              heads over positions [0, position] of the session's cache
//   GEMM       o = att W_o^T
//   add_ln     x += o; LN_xq(x)
//   GEMM       q_x = LN_xq(x) W_xq^T                  (one 128-wide head)
//   cross_attn attention over the session's text keys with the condition
//              mask, renormalised by the alignment prior on layers 2..10;
//              layers 4, 5, 8, 9 keep their probabilities, layer 9 writes
//              their mean (the alignment scores)
//   GEMM       o = ctx W_xo^T
//   add_ln     x += o; LN_ff(x)
//   GEMM+gelu  h = GELU(bf16(LN_ff(x) W_ffn1^T))      (GELU in the GEMM's epilogue)
//   GEMM       o = h W_ffn2^T                          (K split in 4: f32 partial sums)
//   add_ln     x += bf16(sum of the partials); LN of the next layer (or the output norm)
// The GEMMs run on gemm_tc.cuh's persistent tcgen05 kernel with the 2 x
// sessions activation rows on the MMA's M side (128 per tile) and the output
// features on its N side (256 per tile, the full-rate shape).  The self-attention
// cache stream is the step's dominant traffic (keys and values of every
// layer, head and CFG row up to the position), so that kernel is written for
// HBM bandwidth: one CTA per (session, row, head), keys and values streamed
// together in one pass through a shared-memory ring filled by bulk copies.
#include <map>
#include <mutex>
#include <tuple>

#include "../../include/magpie_tts_rt_b200.h"
#include "common.cuh"
#include "eos_proj.cuh"
#include "gemm_tc.cuh"

namespace mtt {
namespace {

using bf16 = __nv_bfloat16;

constexpr int kW = 768;          // model width
constexpr int kMH = 12;          // self-attention heads
constexpr int kMD = 64;          // self-attention head width
constexpr int kXD = 128;         // cross-attention head width (one head)
constexpr int kFF = 3072;        // FFN width
constexpr int kQKV = 3 * kW;
constexpr int kMaxText = 512;
constexpr int kAlignSlots = 4;
constexpr int kLnThreads = 128;  // 4 rows per CTA, one warp per row

__device__ __forceinline__ float bfr(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ void unpack8f(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = __bfloat1622float2(h[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8f(const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162 h[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
  u.x = *reinterpret_cast<uint32_t*>(&h[0]);
  u.y = *reinterpret_cast<uint32_t*>(&h[1]);
  u.z = *reinterpret_cast<uint32_t*>(&h[2]);
  u.w = *reinterpret_cast<uint32_t*>(&h[3]);
  return u;
}

struct Step {
  int n, L, cap, S;
  const bf16 *pos, *ln_self, *qkv_w, *o_w, *ln_xq, *xq_w, *xo_w, *ln_ff, *ffn1_w, *ffn2_w, *norm_out;
  const bf16* embedded;
  const int64_t* position;
  const uint32_t* text_length;
  const bool* active;
  bf16 *self_k, *self_v;
  bool* self_mask;
  const bf16 *cross_k, *cross_v;
  const bool* cond_mask;
  const bf16* prior;
  bf16* hidden;
  bf16* alignment;
  int32_t* status;
  // workspace
  bf16 *x, *ln, *qkv, *att, *o, *xq, *ctx, *h, *align;
  float* part;  // split-K partial sums [splits][2n][768] of the GEMM before an add_ln
};

__device__ __forceinline__ bool session_active(const Step& st, int s) {
  return st.active == nullptr || st.active[s];
}

__device__ __forceinline__ bool session_live(const Step& st, int s) {
  if (!session_active(st, s)) return false;
  const int64_t p = st.position[s];
  const uint32_t t = st.text_length[s];
  return p >= 0 && p < st.cap && t >= 1 && t <= static_cast<uint32_t>(st.S);
}

// ---------------------------------------------------------------------------
// x = bf16(x + o), then LN(x) with the weight (no bias, eps 1e-5): one warp
// per row of 768 (24 values per lane, two passes for the variance).  kEmbed:
// layer 0's input instead, x = bf16(embedded[s] + pos[position[s]]) for both
// rows of session s (main_decoder_wrapper.py:826-829), and the session's
// status.  `out` receives the normalised row; rows of sessions that are
// inactive or out of range are left as they are.
// ---------------------------------------------------------------------------
template <bool kEmbed>
__global__ void __launch_bounds__(kLnThreads) add_ln_kernel(Step st, const bf16* __restrict__ w, bf16* out,
                                                            int partials) {
  // one wave of small CTAs: let the next GEMM set up and fetch its weights meanwhile
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  wait_prior_grid();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (kLnThreads / 32) + (threadIdx.x >> 5);
  if (row >= 2 * st.n) return;
  const int s = row >> 1;
  if (kEmbed && lane == 0 && (row & 1) == 0 && session_active(st, s)) st.status[s] = session_live(st, s) ? 0 : 1;
  if (!session_live(st, s)) return;
  float v[24];
  bf16* xr = st.x + static_cast<size_t>(row) * kW;
  uint4 wq[3];  // the LayerNorm weights, loaded with the inputs (no dependent load later)
#pragma unroll
  for (int c = 0; c < 3; ++c) wq[c] = *reinterpret_cast<const uint4*>(w + 8 * (lane + 32 * c));
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const int col = 8 * (lane + 32 * c);
    float a[8], b[8];
    if (kEmbed) {
      unpack8f(*reinterpret_cast<const uint4*>(st.embedded + static_cast<size_t>(s) * kW + col), a);
      unpack8f(*reinterpret_cast<const uint4*>(st.pos + static_cast<size_t>(st.position[s]) * kW + col), b);
    } else if (partials > 0) {
      // the split GEMM's output: its partial sums in split order, rounded once to bf16
      unpack8f(*reinterpret_cast<const uint4*>(xr + col), a);
#pragma unroll
      for (int e = 0; e < 8; ++e) b[e] = 0.f;
      for (int ks = 0; ks < partials; ++ks) {
        const float4* pp =
            reinterpret_cast<const float4*>(st.part + (static_cast<size_t>(ks) * 2 * st.n + row) * kW + col);
        const float4 p0 = pp[0], p1 = pp[1];
        b[0] += p0.x; b[1] += p0.y; b[2] += p0.z; b[3] += p0.w;
        b[4] += p1.x; b[5] += p1.y; b[6] += p1.z; b[7] += p1.w;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) b[e] = bfr(b[e]);
    } else {
      unpack8f(*reinterpret_cast<const uint4*>(xr + col), a);
      unpack8f(*reinterpret_cast<const uint4*>(st.o + static_cast<size_t>(row) * kW + col), b);
    }
    float t[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      t[e] = bfr(a[e] + b[e]);
      v[8 * c + e] = t[e];
    }
    *reinterpret_cast<uint4*>(xr + col) = pack8f(t);
  }
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < 24; ++i) sum += v[i];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  const float mean = sum * (1.0f / kW);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < 24; ++i) {
    const float d = v[i] - mean;
    sq += d * d;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
  const float rstd = 1.0f / sqrtf(sq * (1.0f / kW) + 1e-5f);
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const int col = 8 * (lane + 32 * c);
    float g[8], y[8];
    unpack8f(wq[c], g);
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = (v[8 * c + e] - mean) * rstd * g[e];
    *reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * kW + col) = pack8f(y);
  }
}

// ---------------------------------------------------------------------------
// Self-attention of one (session, row, head) over positions [0, p]
// (main_decoder_wrapper.py:836-877 and :188-228): the step's key and value
// are written at position p of the cache first (torch.where on the cache
// position); scores bf16(bf16(q.k) * 1/8), masked by the key mask (position p
// itself is always valid: the step's query mask is all ones), softmax and the
// probability-weighted sum of the values in one pass over the cache (running
// maximum and sum per 8-lane group, rescaled once per four keys, merged at
// the end), rounded to bf16 once.  The probabilities are not rounded to bf16
// before the value sum, as the reference's two separate operations do: one
// rounding fewer, no further from the exact result.
//
// The cache rows [0, p) stream through a two-stage shared-memory ring of
// 64-key chunks (8 KB of keys + 8 KB of values per stage), filled by 1-D bulk
// copies (cp.async.bulk, no multicast) that one thread issues and an mbarrier
// per stage completes; the copies need no registers, so six CTAs per SM keep
// up to 12 chunks in flight (two stages measured 4% faster per decoder step
// than three or four: more CTAs per SM beat deeper rings).  Eight lanes read one 128-byte row from shared
// memory.  A wait that does not complete within its bound marks the session's
// status 2; the kernel then stops issuing and waits (bounded) for the copies
// it issued before it exits.
// ---------------------------------------------------------------------------
constexpr int kSAThreads = 128;
constexpr int kSAGroups = kSAThreads / 8;  // 8-lane groups, one key row each per step
constexpr int kSAChunk = 64;               // keys per stage
constexpr int kSAStages = 2;
constexpr uint32_t kSARowBytes = kMD * 2;  // 128 bytes per key or value row

struct SAStage {
  bf16 k[kSAChunk * kMD];
  bf16 v[kSAChunk * kMD];
};
constexpr size_t kSASmem = kSAStages * sizeof(SAStage);  // 32 KB

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, unsigned long long* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))), "l"(src), "r"(bytes),
               "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
               : "memory");
}

__device__ __forceinline__ bool sa_wait(unsigned long long* bar, uint32_t parity) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
  unsigned long long t0;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t0));
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    if (t - t0 > 20000000ull) return false;  // 20 ms
  }
}

// Running softmax state of an 8-lane group: maximum, sum of exponentials
// and the lane's eight dimensions of the weighted value sum.
struct SARun {
  float m, l;
  float acc[8];
};

__global__ void __launch_bounds__(kSAThreads) self_attn_kernel(Step st, int l) {
  extern __shared__ __align__(128) unsigned char sa_dyn[];
  SAStage* stage = reinterpret_cast<SAStage*>(sa_dyn);
  __shared__ unsigned long long full[kSAStages];
  __shared__ float qs[kMD];
  __shared__ __align__(16) bf16 kn[kMD];
  __shared__ __align__(16) bf16 vn[kMD];
  __shared__ float gm[kSAGroups], gl[kSAGroups];
  __shared__ float gacc[kSAGroups][kMD];
  __shared__ int err, issued;
  wait_prior_grid();
  const int h = blockIdx.x, r = blockIdx.y, s = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = 2 * s + r;
  bf16* out = st.att + static_cast<size_t>(row) * kW + h * kMD;
  if (!session_live(st, s)) {
    if (session_active(st, s) && tid < kMD) out[tid] = __float2bfloat16_rn(0.f);
    return;
  }
  const int p = static_cast<int>(st.position[s]);
  const bf16* qkv = st.qkv + static_cast<size_t>(row) * kQKV;
  const size_t cbase = ((((static_cast<size_t>(s) * st.L + l) * 2 + r) * kMH + h) * st.cap) * kMD;
  bf16* K = st.self_k + cbase;
  bf16* V = st.self_v + cbase;
  bool* mrow = st.self_mask + (static_cast<size_t>(s) * 2 + r) * st.cap;
  const int nchunks = (p + kSAChunk - 1) / kSAChunk;  // cache rows [0, p)
  auto issue = [&](int c) {  // thread 0
    const uint32_t rows = static_cast<uint32_t>(min(kSAChunk, p - kSAChunk * c));
    SAStage& sg = stage[c % kSAStages];
    unsigned long long* bar = &full[c % kSAStages];
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar))), "r"(2 * rows * kSARowBytes)
                 : "memory");
    bulk_load(sg.k, K + static_cast<size_t>(kSAChunk) * c * kMD, rows * kSARowBytes, bar);
    bulk_load(sg.v, V + static_cast<size_t>(kSAChunk) * c * kMD, rows * kSARowBytes, bar);
    issued = c + 1;
  };
  if (tid == 0) {
    err = 0;
    issued = 0;
#pragma unroll
    for (int i = 0; i < kSAStages; ++i)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(&full[i])))
                   : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int c = 0; c < min(kSAStages, nchunks); ++c) issue(c);
  }
  // updated_mask (main_decoder_wrapper.py:853): the step's position joins the
  // keys; no CTA reads mrow[p] (position p counts as valid below)
  if (l == 0 && h == 0 && tid == 0) mrow[p] = true;
  if (tid < kMD) {
    qs[tid] = __bfloat162float(qkv[h * kMD + tid]);
    const bf16 k = qkv[kW + h * kMD + tid], v = qkv[2 * kW + h * kMD + tid];
    kn[tid] = k;
    vn[tid] = v;
    K[static_cast<size_t>(p) * kMD + tid] = k;
    V[static_cast<size_t>(p) * kMD + tid] = v;
  }
  __syncthreads();
  const int sub = lane & 7, slot = lane >> 3;  // 16-byte chunk of a row, row within the warp's four
  const int group = warp * 4 + slot;
  float q8[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) q8[e] = qs[8 * sub + e];
  SARun run{-CUDART_INF_F, 0.f, {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}};
  // fold up to four keys (scores sc[u], valid[u], value rows vr[u]) into the run
  auto fold4 = [&](const float (&sc)[4], const bool (&ok)[4], const uint4 (&vr)[4]) {
    float mn = run.m;
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (ok[u]) mn = fmaxf(mn, sc[u]);
    if (mn == -CUDART_INF_F) return;  // no valid key yet
    const float c = __expf(run.m - mn);
    run.l *= c;
#pragma unroll
    for (int e = 0; e < 8; ++e) run.acc[e] *= c;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (ok[u]) {
        const float ej = __expf(sc[u] - mn);
        float v8[8];
        unpack8f(vr[u], v8);
        run.l += ej;
#pragma unroll
        for (int e = 0; e < 8; ++e) run.acc[e] = fmaf(ej, v8[e], run.acc[e]);
      }
    }
    run.m = mn;
  };
  for (int c = 0; c < nchunks; ++c) {
    const SAStage& sg = stage[c % kSAStages];
    if (!sa_wait(&full[c % kSAStages], static_cast<uint32_t>((c / kSAStages) & 1))) err = 1;
    const int rows = min(kSAChunk, p - kSAChunk * c);
    float sc[4];
    bool ok[4];
    uint4 vr[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int jj = warp * 16 + 4 * u + slot;
      const bool in = jj < rows;
      const uint4 kr = in ? *reinterpret_cast<const uint4*>(sg.k + jj * kMD + 8 * sub) : make_uint4(0, 0, 0, 0);
      vr[u] = in ? *reinterpret_cast<const uint4*>(sg.v + jj * kMD + 8 * sub) : make_uint4(0, 0, 0, 0);
      float k8[8];
      unpack8f(kr, k8);
      float d = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) d = fmaf(q8[e], k8[e], d);
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      d += __shfl_xor_sync(0xffffffffu, d, 4);
      sc[u] = bfr(bfr(d) * 0.125f);
      ok[u] = in && mrow[kSAChunk * c + jj];
    }
    fold4(sc, ok, vr);
    __syncthreads();  // every thread is done with this stage
    if (tid == 0 && err == 0 && c + kSAStages < nchunks) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(c + kSAStages);
    }
  }
  // position p: the step's own key and value, from shared memory (group 0)
  {
    const uint4 kr = *reinterpret_cast<const uint4*>(kn + 8 * sub);
    float k8[8];
    unpack8f(kr, k8);
    float d = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) d = fmaf(q8[e], k8[e], d);
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    d += __shfl_xor_sync(0xffffffffu, d, 2);
    d += __shfl_xor_sync(0xffffffffu, d, 4);
    const float sc[4] = {bfr(bfr(d) * 0.125f), 0.f, 0.f, 0.f};
    const bool ok[4] = {group == 0, false, false, false};
    const uint4 vr[4] = {*reinterpret_cast<const uint4*>(vn + 8 * sub), make_uint4(0, 0, 0, 0),
                         make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
    fold4(sc, ok, vr);
  }
  if (sub == 0) {
    gm[group] = run.m;
    gl[group] = run.l;
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) gacc[group][8 * sub + e] = run.acc[e];
  __syncthreads();
  if (tid == 0 && err != 0) {
    // a wait gave up: wait (bounded) for every copy this CTA issued, then flag the session
    for (int c = max(0, issued - kSAStages); c < issued; ++c)
      sa_wait(&full[c % kSAStages], static_cast<uint32_t>((c / kSAStages) & 1));
    st.status[s] = 2;
  }
  if (tid < kMD) {
    float mx = gm[0];
#pragma unroll
    for (int g = 1; g < kSAGroups; ++g) mx = fmaxf(mx, gm[g]);  // finite: position p is valid
    float L = 0.f, o = 0.f;
#pragma unroll
    for (int g = 0; g < kSAGroups; ++g) {
      const float c = gm[g] == -CUDART_INF_F ? 0.f : __expf(gm[g] - mx);  // 0 for a group without keys
      L = fmaf(gl[g], c, L);
      o = fmaf(gacc[g][tid], c, o);
    }
    out[tid] = __float2bfloat16_rn(o / L);
  }
}

// ---------------------------------------------------------------------------
// Cross-attention of one (session, row) (main_decoder_wrapper.py:559-603,
// :101-122, :293-309): scores bf16(bf16(q.k) * 128^-1/2) over the session's T
// text keys, condition-masked, softmax rounded to bf16; on prior layers
// p = bf16(n / bf16(sum n)) with n = bf16(p * bf16(prior + tiny)); the context
// is the probability-weighted sum of the values.  Alignment layers keep p
// (slots 0..2) and the last writes bf16(mean of the four) (:325-345).
// Sixteen lanes per 256-byte key row, two rows per warp per step.
// ---------------------------------------------------------------------------
constexpr int kXAThreads = 256;

__global__ void __launch_bounds__(kXAThreads) cross_attn_kernel(Step st, int l, int prior_layer, int align_slot) {
  __shared__ float sc[kMaxText];
  __shared__ float qs[kXD];
  __shared__ float part[kXAThreads / 32][kXD];
  __shared__ float red[kXAThreads / 32];
  wait_prior_grid();
  const int r = blockIdx.x, s = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = 2 * s + r;
  bf16* out = st.ctx + static_cast<size_t>(row) * kXD;
  if (!session_live(st, s)) {
    if (session_active(st, s) && tid < kXD) out[tid] = __float2bfloat16_rn(0.f);
    return;
  }
  const int T = static_cast<int>(st.text_length[s]);
  const size_t kb = ((static_cast<size_t>(s) * st.L + l) * 2 + r) * st.S * kXD;
  const bf16* K = st.cross_k + kb;
  const bf16* V = st.cross_v + kb;
  const size_t rb = (static_cast<size_t>(s) * 2 + r) * st.S;
  const bool* cm = st.cond_mask + rb;
  if (tid < kXD) qs[tid] = __bfloat162float(st.xq[static_cast<size_t>(row) * kXD + tid]);
  __syncthreads();
  const int sub = lane & 15, slot = lane >> 4;
  float q8[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) q8[e] = qs[8 * sub + e];
  const float scale = 0.08838834764831845f;  // 128 ** -0.5
  for (int base = warp * 8; base < T; base += 64) {
    uint4 kv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = base + 2 * u + slot;
      kv[u] = j < T ? *reinterpret_cast<const uint4*>(K + static_cast<size_t>(j) * kXD + 8 * sub)
                    : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = base + 2 * u + slot;
      float k8[8];
      unpack8f(kv[u], k8);
      float d = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) d = fmaf(q8[e], k8[e], d);
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
      if (sub == 0 && j < T) sc[j] = cm[j] ? bfr(bfr(d) * scale) : -CUDART_INF_F;
    }
  }
  __syncthreads();
  float m = -CUDART_INF_F;
  for (int j = tid; j < T; j += kXAThreads) m = fmaxf(m, sc[j]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int w = 1; w < kXAThreads / 32; ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  float sum = 0.f;
  for (int j = tid; j < T; j += kXAThreads) {
    const float e = m == -CUDART_INF_F ? 0.f : expf(sc[j] - m);
    sc[j] = e;
    sum += e;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if (lane == 0) red[warp] = sum;
  __syncthreads();
  sum = 0.f;
#pragma unroll
  for (int w = 0; w < kXAThreads / 32; ++w) sum += red[w];
  __syncthreads();
  float nsum = 0.f;
  const bf16* pr = st.prior + rb;
  for (int j = tid; j < T; j += kXAThreads) {
    float pj = cm[j] ? bfr(sc[j] / sum) : 0.f;  // softmax, then masked_fill(~valid, 0)
    if (prior_layer) {
      const float pri = bfr(__bfloat162float(pr[j]) + 1.17549435e-38f);  // prior + finfo(bf16).tiny
      pj = bfr(pj * pri);
      nsum += pj;
    }
    sc[j] = pj;
  }
  if (prior_layer) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) nsum += __shfl_xor_sync(0xffffffffu, nsum, off);
    if (lane == 0) red[warp] = nsum;
    __syncthreads();
    nsum = 0.f;
#pragma unroll
    for (int w = 0; w < kXAThreads / 32; ++w) nsum += red[w];
    const float den = bfr(nsum);
    for (int j = tid; j < T; j += kXAThreads) sc[j] = bfr(sc[j] / den);
  }
  __syncthreads();
  if (align_slot >= 0) {
    for (int j = tid; j < T; j += kXAThreads) {
      if (align_slot < kAlignSlots - 1) {
        st.align[(static_cast<size_t>(align_slot) * 2 * st.n + row) * st.S + j] = __float2bfloat16_rn(sc[j]);
      } else {
        // stack(...).mean(dim=1): the four layers' values summed in layer order, then / 4
        const float a0 = __bfloat162float(st.align[(static_cast<size_t>(0) * 2 * st.n + row) * st.S + j]);
        const float a1 = __bfloat162float(st.align[(static_cast<size_t>(1) * 2 * st.n + row) * st.S + j]);
        const float a2 = __bfloat162float(st.align[(static_cast<size_t>(2) * 2 * st.n + row) * st.S + j]);
        st.alignment[rb + j] = __float2bfloat16_rn((((a0 + a1) + a2) + sc[j]) * 0.25f);
      }
    }
  }
  // context
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int base = warp * 8; base < T; base += 64) {
    uint4 vv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = base + 2 * u + slot;
      vv[u] = j < T ? *reinterpret_cast<const uint4*>(V + static_cast<size_t>(j) * kXD + 8 * sub)
                    : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = base + 2 * u + slot;
      if (j < T) {
        const float pj = sc[j];
        float v8[8];
        unpack8f(vv[u], v8);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(pj, v8[e], acc[e]);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], 16);
  if (slot == 0) {
#pragma unroll
    for (int e = 0; e < 8; ++e) part[warp][8 * sub + e] = acc[e];
  }
  __syncthreads();
  if (tid < kXD) {
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < kXAThreads / 32; ++w) o += part[w][tid];
    out[tid] = __float2bfloat16_rn(o);
  }
}

// ---------------------------------------------------------------------------
// GEMM epilogues (gemm_tc.cuh): lane = output feature m, columns = rows n
// ---------------------------------------------------------------------------

// The EOS projection's bounded waits gave up: its outputs are unreliable, as
// a cache copy that timed out would make them (status 2).
__global__ void eos_status_kernel(Step st, const int32_t* eos_status) {
  wait_prior_grid();
  if (*eos_status == 0) return;
  for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < st.n; s += gridDim.x * blockDim.x) {
    if (session_live(st, s)) st.status[s] = 2;
  }
}

// The projection GEMMs put the activation rows on the MMA's M side (128 per
// tile) and the output features on its N side (256 per tile; 128 for the
// 128-wide cross-attention query): a tcgen05.mma of M = 128, K = 16 costs the
// same for every N up to 256, so N = 256 is the full-rate shape, and each
// epilogue lane then holds 32 consecutive output features of its own row,
// which leave as four 16-byte stores.

// C[m][n] = bf16(D), or GELU-tanh of the bf16-rounded D (the reference rounds
// the FFN1 output before its activation, text_encoder_wrapper.py:61-70).
// Each lane holds 64 bytes of its own row per chunk; the warp stages its 32
// rows in shared memory (row stride 80 bytes: conflict-free 16-byte access)
// and writes them back four lanes per row, so each store instruction covers
// eight whole 64-byte row segments instead of 32 scattered 16-byte pieces.
constexpr int kStageRowB = 40;  // bf16 per staged row (64 bytes + 16 of padding)
struct EpiRows {
  bf16* c;
  int ldc;
  int rows;
  int gelu;
  __device__ __forceinline__ void chunk(int m, int n0, int /*ks*/, const uint32_t (&v)[32], int /*n_cols*/) const {
    __shared__ __align__(16) bf16 stage[kGemmEpiWarps][32][kStageRowB];
    const int lane = threadIdx.x & 31, w = gemm_epi_warp();
    uint32_t packed[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float a = __uint_as_float(v[2 * j]), b = __uint_as_float(v[2 * j + 1]);
      if (gelu) {
        a = bfr(a);
        b = bfr(b);
        a = 0.5f * a * (1.0f + tanhf(0.7978845608028654f * (a + 0.044715f * a * a * a)));
        b = 0.5f * b * (1.0f + tanhf(0.7978845608028654f * (b + 0.044715f * b * b * b)));
      }
      const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
      packed[j] = *reinterpret_cast<const uint32_t*>(&h);
    }
    uint4* mine = reinterpret_cast<uint4*>(stage[w][lane]);
#pragma unroll
    for (int q = 0; q < 4; ++q) mine[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
    __syncwarp();
    const int m0 = m - lane;  // the warp's first row
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int r = 8 * it + (lane >> 2), q = lane & 3;
      if (m0 + r < rows) {
        reinterpret_cast<uint4*>(c + static_cast<size_t>(m0 + r) * ldc + n0)[q] =
            reinterpret_cast<const uint4*>(stage[w][r])[q];
      }
    }
    __syncwarp();
  }
};

// part[ks][m][n] = D of split ks (f32), summed by the next add_ln_kernel;
// staged like EpiRows, 16 columns (64 bytes per row) at a time.
constexpr int kStageRowF = 20;  // f32 per staged row (64 bytes + 16 of padding)
struct EpiPartial {
  float* part;
  int ldc;
  int rows;
  size_t split_stride;
  __device__ __forceinline__ void chunk(int m, int n0, int ks, const uint32_t (&v)[32], int /*n_cols*/) const {
    __shared__ __align__(16) float stage[kGemmEpiWarps][32][kStageRowF];
    const int lane = threadIdx.x & 31, w = gemm_epi_warp();
    const int m0 = m - lane;
    float* base = part + static_cast<size_t>(ks) * split_stride;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float4* mine = reinterpret_cast<float4*>(stage[w][lane]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        mine[q] = make_float4(__uint_as_float(v[16 * h + 4 * q]), __uint_as_float(v[16 * h + 4 * q + 1]),
                              __uint_as_float(v[16 * h + 4 * q + 2]), __uint_as_float(v[16 * h + 4 * q + 3]));
      }
      __syncwarp();
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int r = 8 * it + (lane >> 2), q = lane & 3;
        if (m0 + r < rows) {
          reinterpret_cast<float4*>(base + static_cast<size_t>(m0 + r) * ldc + n0 + 16 * h)[q] =
              reinterpret_cast<const float4*>(stage[w][r])[q];
        }
      }
      __syncwarp();
    }
  }
};

// FFN2 (K = 3072) splits its K range in 4 (12 chunks of 64 each, as long as
// the other GEMMs' K = 768); add_ln_kernel sums the f32 partials.  Splitting
// the K = 768 GEMMs as well measured slower (the partials' traffic costs more
// than the shorter K range saves).
constexpr int kFfn2Splits = 4;
constexpr int kMaxSplits = kFfn2Splits;

// C[rows][N] = X[rows][K] W[N][K]^T on the tensor cores (K a multiple of
// 64 x splits, N of 128); with partial != nullptr the K range is split in
// `splits` and the f32 partial sums go to partial[split][rows][N].
// The weight tile (N side) is the narrowest of 256 / 128 / 64 columns that
// keeps every tile in one wave of the SMs: at 512 activation rows a 256-wide
// tile leaves 12 of the 148 SMs to the 768 x 768 projections, each streaming
// ~590 KB, where 64-wide tiles give 48 CTAs streaming ~290 KB each and MMAs
// of N = 64 (~48 cycles against ~128 at N = 256).
int gemm_weight_tile(int rows, int N, int splits) {
  const int m_tiles = (rows + 127) / 128;
  const int sms = gemm_grid(1 << 30);  // the device's SM count (0 when unknown)
  int bn = N % 256 == 0 ? 256 : 128;
  for (const int cand : {128, 64}) {
    if (cand < bn && N % cand == 0 && m_tiles * (N / cand) * splits <= sms) bn = cand;
  }
  return bn;
}

bool tc_gemm(const bf16* X, const bf16* W, bf16* C, int rows, int N, int K, bool gelu, int splits, float* partial,
             cudaStream_t stream) {
  const int bn = gemm_weight_tile(rows, N, partial != nullptr ? splits : 1);
  CUtensorMap amap, bmap;
  if (!cached_map(&amap, X, static_cast<uint64_t>(K), static_cast<uint64_t>(rows), 128) ||
      !cached_map(&bmap, W, static_cast<uint64_t>(K), static_cast<uint64_t>(N), static_cast<uint32_t>(bn))) {
    return false;
  }
  GemmProblem pr;
  pr.m_tiles = (rows + 127) / 128;
  pr.m_rows_dev = nullptr;
  pr.m_rows_scale = 1;
  pr.n_rows = N;
  pr.n_rows_dev = nullptr;
  pr.n_rows_scale = 1;
  pr.splits = partial != nullptr ? splits : 1;
  pr.k_chunks = K / kGemmKChunk / pr.splits;
  pr.status = nullptr;
  pr.b_constant = 1;  // the weights: fetched while the previous kernel finishes
  cudaError_t e;
  if (partial != nullptr) {
    EpiPartial epi{partial, N, rows, static_cast<size_t>(rows) * N};
    e = bn == 64    ? launch_gemm_tc<64>(amap, bmap, pr, epi, stream)
        : bn == 128 ? launch_gemm_tc<128>(amap, bmap, pr, epi, stream)
                    : launch_gemm_tc<256>(amap, bmap, pr, epi, stream);
  } else {
    EpiRows epi{C, N, rows, gelu ? 1 : 0};
    e = bn == 64    ? launch_gemm_tc<64>(amap, bmap, pr, epi, stream)
        : bn == 128 ? launch_gemm_tc<128>(amap, bmap, pr, epi, stream)
                    : launch_gemm_tc<256>(amap, bmap, pr, epi, stream);
  }
  return e == cudaSuccess;
}

struct MdLayout {
  size_t x, ln, qkv, att, o, xq, ctx, h, align, part, eos_status, total;
};

MdLayout md_layout(int n, int S) {
  MdLayout lo{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off += (bytes + 255) & ~static_cast<size_t>(255);
    return at;
  };
  const size_t rows = 2 * static_cast<size_t>(n);
  lo.x = take(rows * kW * 2);
  lo.ln = take(rows * kW * 2);
  lo.qkv = take(rows * kQKV * 2);
  lo.att = take(rows * kW * 2);
  lo.o = take(rows * kW * 2);
  lo.xq = take(rows * kXD * 2);
  lo.ctx = take(rows * kXD * 2);
  lo.h = take(rows * kFF * 2);
  lo.align = take((kAlignSlots - 1) * rows * S * 2);
  lo.part = take(static_cast<size_t>(kMaxSplits) * rows * kW * 4);
  lo.eos_status = take(4);
  lo.total = off;
  return lo;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Every kernel of the step is launched with programmatic stream serialization
// (common.cuh): its CTAs may be scheduled while the previous launch on the
// stream (a library GEMM, say) drains, and each kernel calls wait_prior_grid()
// before its first global memory access.
template <typename... KArgs, typename... Args>
bool launch_after(void (*kernel)(KArgs...), dim3 grid, unsigned block, size_t smem, cudaStream_t stream,
                  Args... args) {
  return launch_serialized(kernel, grid, dim3(block, 1, 1), smem, stream, args...) == cudaSuccess;
}

}  // namespace
}  // namespace mtt

extern "C" MTT_B200_API size_t mtt_b200_main_decoder_workspace_size(int32_t max_sessions, int32_t token_stride) {
  if (max_sessions <= 0 || token_stride <= 0 || token_stride > mtt::kMaxText || token_stride % 8 != 0) return 0;
  return mtt::md_layout(max_sessions, token_stride).total;
}

extern "C" MTT_B200_API int mtt_b200_launch_main_decoder_step(const mtt_b200_main_decoder_weights_t* w,
                                                             const mtt_b200_main_decoder_batch_t* b, void* workspace,
                                                             size_t workspace_bytes, void* stream) {
  using namespace mtt;
  if (w == nullptr || b == nullptr || workspace == nullptr || b->n_sessions <= 0 || w->n_layers < 10 ||
      b->cache_capacity <= 0 || b->token_stride <= 0 || b->token_stride > kMaxText || b->token_stride % 8 != 0) {
    return MTT_B200_STATUS_INVALID_ARGUMENT;
  }
  if (!w->pos || !w->ln_self || !w->qkv || !w->o || !w->ln_xq || !w->xq || !w->xo || !w->ln_ff || !w->ffn1 ||
      !w->ffn2 || !w->norm_out || w->pos_rows < b->cache_capacity) {
    return MTT_B200_STATUS_INVALID_ARGUMENT;
  }
  if (!b->embedded || !b->position || !b->text_length || !b->self_k || !b->self_v || !b->self_mask || !b->cross_k ||
      !b->cross_v || !b->cond_mask || !b->prior || !b->hidden || !b->alignment || !b->status) {
    return MTT_B200_STATUS_INVALID_ARGUMENT;
  }
  if (b->eos_projection != nullptr && (w->final_w == nullptr || w->final_b == nullptr || !aligned16(w->final_w) ||
                                      !aligned16(b->eos_projection))) {
    return MTT_B200_STATUS_INVALID_ARGUMENT;
  }
  const void* vec[] = {b->embedded, b->self_k, b->self_v, b->cross_k, b->cross_v, b->hidden, w->pos, w->ln_self,
                       w->ln_xq, w->ln_ff, w->norm_out};
  for (const void* p : vec)
    if (!aligned16(p)) return MTT_B200_STATUS_INVALID_ARGUMENT;
  const MdLayout lo = md_layout(b->n_sessions, b->token_stride);
  if (workspace_bytes < lo.total || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return MTT_B200_STATUS_INVALID_ARGUMENT;
  const cudaStream_t cs = static_cast<cudaStream_t>(stream);

  Step st{};
  st.n = b->n_sessions;
  st.L = w->n_layers;
  st.cap = b->cache_capacity;
  st.S = b->token_stride;
  auto B = [](const void* p) { return static_cast<const bf16*>(p); };
  st.pos = B(w->pos);
  st.ln_self = B(w->ln_self);
  st.qkv_w = B(w->qkv);
  st.o_w = B(w->o);
  st.ln_xq = B(w->ln_xq);
  st.xq_w = B(w->xq);
  st.xo_w = B(w->xo);
  st.ln_ff = B(w->ln_ff);
  st.ffn1_w = B(w->ffn1);
  st.ffn2_w = B(w->ffn2);
  st.norm_out = B(w->norm_out);
  st.embedded = B(b->embedded);
  st.position = b->position;
  st.text_length = b->text_length;
  st.active = b->active;
  st.self_k = static_cast<bf16*>(b->self_k);
  st.self_v = static_cast<bf16*>(b->self_v);
  st.self_mask = b->self_mask;
  st.cross_k = B(b->cross_k);
  st.cross_v = B(b->cross_v);
  st.cond_mask = b->cond_mask;
  st.prior = B(b->prior);
  st.hidden = static_cast<bf16*>(b->hidden);
  st.alignment = static_cast<bf16*>(b->alignment);
  st.status = b->status;
  char* ws = static_cast<char*>(workspace);
  st.x = reinterpret_cast<bf16*>(ws + lo.x);
  st.ln = reinterpret_cast<bf16*>(ws + lo.ln);
  st.qkv = reinterpret_cast<bf16*>(ws + lo.qkv);
  st.att = reinterpret_cast<bf16*>(ws + lo.att);
  st.o = reinterpret_cast<bf16*>(ws + lo.o);
  st.xq = reinterpret_cast<bf16*>(ws + lo.xq);
  st.ctx = reinterpret_cast<bf16*>(ws + lo.ctx);
  st.h = reinterpret_cast<bf16*>(ws + lo.h);
  st.align = reinterpret_cast<bf16*>(ws + lo.align);
  st.part = reinterpret_cast<float*>(ws + lo.part);

  const int M = 2 * st.n;
  const unsigned ln_grid = static_cast<unsigned>((M + kLnThreads / 32 - 1) / (kLnThreads / 32));
  if (cudaFuncSetAttribute(self_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(kSASmem)) != cudaSuccess) {
    return MTT_B200_STATUS_CUDA_ERROR;
  }
  auto layer_w = [](const bf16* base, size_t per_layer, int l) { return base + per_layer * l; };
  if (!launch_after(add_ln_kernel<true>, dim3(ln_grid), kLnThreads, 0, cs, st, st.ln_self, st.ln, 0)) {
    return MTT_B200_STATUS_CUDA_ERROR;
  }
  int slot = 0;
  for (int l = 0; l < st.L; ++l) {
    bool ok = tc_gemm(st.ln, layer_w(st.qkv_w, static_cast<size_t>(kQKV) * kW, l), st.qkv, M, kQKV, kW, false, 1,
                      nullptr, cs);
    ok = ok && launch_after(self_attn_kernel, dim3(kMH, 2, st.n), kSAThreads, kSASmem, cs, st, l);
    ok = ok && tc_gemm(st.att, layer_w(st.o_w, static_cast<size_t>(kW) * kW, l), st.o, M, kW, kW, false, 1, nullptr,
                       cs);
    ok = ok && launch_after(add_ln_kernel<false>, dim3(ln_grid), kLnThreads, 0, cs, st, layer_w(st.ln_xq, kW, l),
                            st.ln, 0);
    ok = ok && tc_gemm(st.ln, layer_w(st.xq_w, static_cast<size_t>(kXD) * kW, l), st.xq, M, kXD, kW, false, 1,
                       nullptr, cs);
    const bool prior_layer = l >= 2 && l <= 10;
    const bool align_layer = l == 4 || l == 5 || l == 8 || l == 9;
    ok = ok && launch_after(cross_attn_kernel, dim3(2, st.n), kXAThreads, 0, cs, st, l, prior_layer ? 1 : 0,
                            align_layer ? slot : -1);
    if (align_layer) ++slot;
    ok = ok && tc_gemm(st.ctx, layer_w(st.xo_w, static_cast<size_t>(kW) * kXD, l), st.o, M, kW, kXD, false, 1,
                       nullptr, cs);
    ok = ok && launch_after(add_ln_kernel<false>, dim3(ln_grid), kLnThreads, 0, cs, st, layer_w(st.ln_ff, kW, l),
                            st.ln, 0);
    ok = ok && tc_gemm(st.ln, layer_w(st.ffn1_w, static_cast<size_t>(kFF) * kW, l), st.h, M, kFF, kW, true, 1,
                       nullptr, cs);
    ok = ok && tc_gemm(st.h, layer_w(st.ffn2_w, static_cast<size_t>(kW) * kFF, l), nullptr, M, kW, kFF, false,
                       kFfn2Splits, st.part, cs);
    const bool last = l + 1 == st.L;
    ok = ok && launch_after(add_ln_kernel<false>, dim3(ln_grid), kLnThreads, 0, cs, st,
                            last ? st.norm_out : layer_w(st.ln_self, kW, l + 1), last ? st.hidden : st.ln,
                            kFfn2Splits);
    if (!ok) return MTT_B200_STATUS_CUDA_ERROR;
  }
  if (b->eos_projection != nullptr) {
    // The Local AR's EOS projection of the hidden state just produced, for
    // every session, on the tensor cores (eos_proj.cuh); the LN buffer is free.
    EosProjArgs ea;
    ea.hidden = st.hidden;
    ea.hidden_stream_stride = 2 * static_cast<int64_t>(kW);
    ea.uncond_offset = kW;
    ea.list = nullptr;
    ea.count = nullptr;
    ea.n_max = st.n;
    ea.weight = static_cast<const bf16*>(w->final_w);
    ea.bias = static_cast<const bf16*>(w->final_b);
    ea.cfg_scale = b->eos_cfg_scale;
    ea.rows = st.ln;
    ea.max_key = static_cast<uint32_t*>(b->eos_projection);
    ea.eos_logit = static_cast<float*>(b->eos_projection) + kPositions;
    ea.proj_stride = 2 * kPositions;
    ea.status = reinterpret_cast<int32_t*>(ws + lo.eos_status);
    if (launch_eos_projection(ea, cs) != cudaSuccess ||
        !launch_after(eos_status_kernel, dim3((st.n + 255) / 256), 256, 0, cs, st,
                      static_cast<const int32_t*>(ea.status))) {
      return MTT_B200_STATUS_CUDA_ERROR;
    }
  }
  return cudaPeekAtLastError() == cudaSuccess ? MTT_B200_STATUS_OK : MTT_B200_STATUS_CUDA_ERROR;
}

extern "C" MTT_B200_API int mtt_b200_launch_test_gemm(const void* x_bf16, const void* w_bf16, void* y_bf16,
                                                     int32_t rows, int32_t n, int32_t k, int32_t gelu, int32_t splits,
                                                     float* partial, void* stream) {
  using namespace mtt;
  if (x_bf16 == nullptr || w_bf16 == nullptr || rows <= 0 || n <= 0 || n % 128 != 0 || k <= 0 || splits <= 0 ||
      k % (kGemmKChunk * splits) != 0 || (splits > 1 ? partial == nullptr : y_bf16 == nullptr)) {
    return MTT_B200_STATUS_INVALID_ARGUMENT;
  }
  const bool ok = tc_gemm(static_cast<const bf16*>(x_bf16), static_cast<const bf16*>(w_bf16),
                          static_cast<bf16*>(y_bf16), rows, n, k, gelu != 0, splits, splits > 1 ? partial : nullptr,
                          static_cast<cudaStream_t>(stream));
  return ok && cudaPeekAtLastError() == cudaSuccess ? MTT_B200_STATUS_OK : MTT_B200_STATUS_CUDA_ERROR;
}
