// Batched decode of libivonar_b200.so: `batch` independent sequences advance one token per step
// together. The projections of all sequences run as one tcgen05 GEMM per matrix (ivb_ternary_gemm over
// `batch` token rows, so the weights stream once per step for the whole batch); the per-sequence parts
// — SSM step, latent-cache append and absorbed latent attention over the sequence's own cache, the
// sampler — run one CTA (or a channel slice) per sequence. The arithmetic of each part is the
// single-sequence decode step's (kernels/ternary.cu:421-482 recurrent_step, :509-611 attention_step,
// :1099-1337 sample_token; decoder.py:235-297 for the torch forms).
#include <cuda_runtime.h>

#include <algorithm>

#include "ivb_common.h"
#include "ivb_decode.cuh"
#include "ivb_tiles.cuh"

extern "C" {
int32_t ivb_quantize_rows(const float* x, int32_t rows, int32_t n, const float* norm_weight, float norm_eps,
                          float norm_clip, float act_eps, int8_t* q8, int32_t ldq, float* scale, int32_t* gsum,
                          void* stream);
int32_t ivb_ternary_gemm(const IvbTernary* m, const int8_t* q8, int32_t ldq, const float* act_scale, int32_t rows_t,
                         int32_t epilogue, float* out, int32_t ldo, uint32_t* error, void* stream);
}

namespace ivb {
namespace {

constexpr int kBatchTaps = 8;  // conv window registers (conv_taps - 1 <= 8)

__global__ void __launch_bounds__(kThreads) batch_embed_kernel(IvbTernary head, const int64_t* tokens, int d, float* resid,
                                                               int32_t* step_counter) {
  const int b = blockIdx.x;
  if (b == 0 && threadIdx.x == 0 && step_counter != nullptr) *step_counter += 1;
  const long long tok = tokens[b];
  const uint8_t* erow = head.packed + static_cast<size_t>(tok) * head.row_bytes;
  const uint16_t* srow = head.scales + static_cast<size_t>(tok) * head.scale_stride;
  for (int i = threadIdx.x; i < d; i += kThreads)
    resid[static_cast<size_t>(b) * d + i] =
        static_cast<float>(((__ldg(erow + (i >> 2)) >> ((i & 3) << 1)) & 3) - 1) * h2f(__ldg(srow + (i >> 7)));
}

// One SSM step of sequence blockIdx.y for 128 consecutive channels (one thread each, so the state of a
// (head, state) row is read and written contiguously across the threads); the per-(head, state)
// coefficients of the heads the CTA touches are computed once into shared memory. ent row b = value |
// gate | per head (B, C, dt). Same arithmetic as the single-sequence decode step, including the order
// of the sum over the states (the xor butterfly of a 16-lane warp sum).
constexpr int kSsmChannels = 128;
__global__ void __launch_bounds__(kSsmChannels) batch_ssm_kernel(IvbLayerDesc L, IvbBatchLayer B, const float* ent, int ld,
                                                                 int d, int H, int hd, int S, int taps, float half_dt_min,
                                                                 float half_dt_range, float* y) {
  extern __shared__ float coef[];  // [heads touched][S][5]: B, C, half_dt, ar, ai
  const int b = blockIdx.y, c0 = blockIdx.x * kSsmChannels;
  const int c = c0 + threadIdx.x;
  const int h0 = c0 / hd, nh = (min(d, c0 + kSsmChannels) - 1) / hd - h0 + 1;
  const float* row = ent + static_cast<size_t>(b) * ld;
  const bool live = c < d;
  const int h = live ? c / hd : h0, dd = live ? c - h * hd : 0;
  float* ssm = B.ssm_state + static_cast<size_t>(b) * H * S * hd * 2;
  float* prevf = B.prev_force + static_cast<size_t>(b) * H * S * hd;
  // this channel's states (every one loaded before the first store, so the loads overlap) and inputs,
  // issued before the coefficients so their latency hides behind the transcendental functions
  float st_r[16], st_i[16], st_p[16];
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    st_r[s] = st_i[s] = st_p[s] = 0.0f;
    if (live && s < S) {
      const size_t si = (static_cast<size_t>(h) * S + s) * hd + dd;
      const float2 v = reinterpret_cast<const float2*>(ssm)[si];
      st_r[s] = v.x;
      st_i[s] = v.y;
      st_p[s] = prevf[si];
    }
  }
  const float incoming = live ? row[c] : 0.0f, gate = live ? row[d + c] : 0.0f;
  for (int i = threadIdx.x; i < nh * S; i += kSsmChannels) {
    const int hh = h0 + i / S, s = i - (i / S) * S;
    const float* bcdt = row + 2 * d + hh * 3 * S;
    const float half_dt = half_dt_min + sigmoid_f(bcdt[2 * S + s]) * half_dt_range;
    const float mag = expf(2.0f * half_dt * L.decay[hh * S + s]);
    float sn, cs;
    sincosf(2.0f * half_dt * L.theta[hh * S + s], &sn, &cs);
    float* cf = coef + i * 5;
    cf[0] = tanhf(bcdt[s]);
    cf[1] = tanhf(bcdt[S + s]);
    cf[2] = half_dt;
    cf[3] = mag * cs;
    cf[4] = mag * sn;
  }
  __syncthreads();
  if (!live) return;
  float* conv_state = B.conv_state + static_cast<size_t>(b) * d * (taps - 1) + static_cast<size_t>(c) * (taps - 1);
  float conv = L.conv_bias[c];
  for (int k2 = 0; k2 < taps - 1; ++k2) conv = fmaf(L.conv_weight[c * taps + k2], conv_state[k2], conv);
  conv = fmaf(L.conv_weight[c * taps + taps - 1], incoming, conv);
  const float value = silu_f(conv);
  float contrib[16];
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    contrib[s] = 0.0f;
    if (s < S) {
      const float* cf = coef + ((h - h0) * S + s) * 5;
      const size_t si = (static_cast<size_t>(h) * S + s) * hd + dd;
      const float sr = st_r[s], sim = st_i[s], prev = st_p[s];
      const float force = cf[0] * value;
      const float dr = (force + cf[3] * prev) * cf[2];
      const float di = (cf[4] * prev) * cf[2];
      const float nr = sr * cf[3] - sim * cf[4] + dr;
      const float ni = sr * cf[4] + sim * cf[3] + di;
      reinterpret_cast<float2*>(ssm)[si] = make_float2(nr, ni);
      prevf[si] = force;
      contrib[s] = cf[1] * nr;
    }
  }
  float a8[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) a8[i] = contrib[i] + contrib[i + 8];
  const float sum = ((a8[0] + a8[4]) + (a8[2] + a8[6])) + ((a8[1] + a8[5]) + (a8[3] + a8[7]));
  y[static_cast<size_t>(b) * d + c] = (sum + L.skip[c] * value) * sigmoid_f(gate);
  // shift the conv window: the oldest input leaves, this token's enters
  for (int k = 0; k + 1 < taps - 1; ++k) conv_state[k] = conv_state[k + 1];
  if (taps > 1) conv_state[taps - 2] = incoming;
}

// Latent-cache append of sequence blockIdx.x at its position: quantised latent + rotated k_rope.
__global__ void __launch_bounds__(kThreads) batch_cache_kernel(IvbLayerDesc L, IvbBatchLayer B, const float* ent, int ld,
                                                               const int64_t* positions, int d, int Lt, int H, int rope,
                                                               int max_len, int lpad, int rpad, float act_eps,
                                                               unsigned* error) {
  __shared__ float xl[512 + 64];
  __shared__ __align__(16) int8_t codes[576];
  __shared__ float red[64];
  const int b = blockIdx.x;
  const long long pos = positions[b];
  if (pos < 0 || pos >= max_len) {
    if (threadIdx.x == 0) atomicCAS(error, 0u, static_cast<unsigned>(IVB_ECAPACITY));
    return;
  }
  const float* row = ent + static_cast<size_t>(b) * ld;
  for (int j = threadIdx.x; j < Lt; j += kThreads) xl[j] = row[d + j];
  __syncthreads();
  const float a = quantize_block(xl, Lt, nullptr, 0.0f, 0.0f, act_eps, codes, false, nullptr, red);
  int8_t* latent_q = B.latent_q + static_cast<size_t>(b) * max_len * lpad;
  for (int j = threadIdx.x; j < Lt; j += kThreads) latent_q[pos * lpad + j] = codes[j];
  if (threadIdx.x == 0) B.latent_scale[static_cast<size_t>(b) * max_len + pos] = a;
  const float* rtab = L.rope + pos * rope;
  uint16_t* kcache = B.k_rope_cache + static_cast<size_t>(b) * H * max_len * rpad;
  for (int i = threadIdx.x; i < H * (rope / 2); i += kThreads) {
    const int h = i / (rope / 2), jr = i - h * (rope / 2);
    const float cs = __ldg(rtab + 2 * jr), sn = __ldg(rtab + 2 * jr + 1);
    const float k0 = row[d + Lt + h * rope + 2 * jr], k1 = row[d + Lt + h * rope + 2 * jr + 1];
    uint16_t* kc = kcache + (static_cast<size_t>(h) * max_len + pos) * rpad;
    kc[2 * jr] = f2h(k0 * cs - k1 * sn);
    kc[2 * jr + 1] = f2h(k0 * sn + k1 * cs);
  }
}

// Absorbed latent attention of sequence blockIdx.x, head blockIdx.y, over cached positions 0..pos:
// s_p = a_p <qa, ql_p> + q_nope.b_k + <q_rope, k_rope_p>, online softmax, out = W_v (sum_p w_p a_p ql_p) + b_v.
constexpr int kAttnThreads = 128;
constexpr int kAttnTile = 128;

__global__ void __launch_bounds__(kAttnThreads) batch_attention_kernel(IvbLayerDesc L, IvbBatchLayer B, const float* ent,
                                                                       int ld, const int64_t* positions, int d, int Lt, int H,
                                                                       int hd, int rope, int nope, int max_len, int lpad,
                                                                       int rpad, float* y) {
  __shared__ float qa[512];
  __shared__ float qn[256];
  __shared__ float qr[128];
  __shared__ float sc[kAttnTile];
  __shared__ float part[4][512];
  __shared__ float red[64];
  const int t = blockIdx.x, h = blockIdx.y;
  const long long pos_in = positions[t];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (pos_in < 0 || pos_in >= max_len) {  // capacity error, reported by the cache append
    for (int e = tid; e < hd; e += kAttnThreads) y[static_cast<size_t>(t) * d + h * hd + e] = 0.0f;
    return;
  }
  const int pos = static_cast<int>(pos_in);
  // sequence t's caches
  const int8_t* latent_q = B.latent_q + static_cast<size_t>(t) * max_len * lpad;
  const float* latent_scale = B.latent_scale + static_cast<size_t>(t) * max_len;
  const uint16_t* k_rope_cache = B.k_rope_cache + static_cast<size_t>(t) * H * max_len * rpad;
  const float* q = ent + static_cast<size_t>(t) * ld + h * hd;
  const float scl = L.attn_scale;
  const float* rtab = L.rope + static_cast<size_t>(pos) * rope;
  for (int jr = tid; jr < rope / 2; jr += kAttnThreads) {
    const float cs = __ldg(rtab + 2 * jr), sn = __ldg(rtab + 2 * jr + 1);
    const float q0 = q[nope + 2 * jr], q1 = q[nope + 2 * jr + 1];
    qr[2 * jr] = (q0 * cs - q1 * sn) * scl;
    qr[2 * jr + 1] = (q0 * sn + q1 * cs) * scl;
  }
  for (int e = tid; e < nope; e += kAttnThreads) qn[e] = q[e] * scl;
  __syncthreads();
  // absorbed query qa[j] = sum_e qn[e] W_k[h nope + e][j]: thread = (e-group, 16-input word of the
  // latent row), the e-groups summed in order through shared memory
  const IvbTernary& kn = L.k_nope_up;
  {
    const int words = (Lt + 15) >> 4, n_eg = kAttnThreads / words;  // n_eg * Lt <= 2048 = part
    float* pe = &part[0][0];
    const int wd = tid % words, eg = tid / words;
    if (eg < n_eg) {
      float acc[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] = 0.0f;
      for (int e = eg; e < nope; e += n_eg) {
        const size_t r = static_cast<size_t>(h) * nope + e;
        const unsigned w = __ldg(reinterpret_cast<const unsigned*>(kn.packed + r * kn.row_bytes) + wd);
        const float qs = qn[e] * h2f(__ldg(kn.scales + r * kn.scale_stride + (wd >> 3)));
        float cm1[16];
        word_codes_m1(w, cm1);
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = fmaf(qs, cm1[i], acc[i]);
      }
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (wd * 16 + i < Lt) pe[eg * Lt + wd * 16 + i] = acc[i];
    }
    __syncthreads();
    for (int j = tid; j < Lt; j += kAttnThreads) {
      float v = pe[j];
      for (int g2 = 1; g2 < n_eg; ++g2) v += pe[g2 * Lt + j];
      qa[j] = v;
    }
  }
  float qb = 0.0f;
  if (kn.bias != nullptr) {
    float pp = 0.0f;
    for (int e = tid; e < nope; e += kAttnThreads) pp = fmaf(qn[e], __ldg(kn.bias + h * nope + e), pp);
    pp = warp_sum(pp);
    if (lane == 0) red[warp] = pp;
    __syncthreads();
    qb = red[0];
    for (int w = 1; w < kAttnThreads / 32; ++w) qb += red[w];
  }
  __syncthreads();
  const int sub = tid & 7, grp = tid >> 3;  // 16 position groups of 8 lanes
  const int P = pos + 1;
  float m_run = -INFINITY, l_run = 0.0f;
  float u[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) u[i] = 0.0f;
  for (int start = 0; start < P; start += kAttnTile) {
    const int count = min(kAttnTile, P - start);
    for (int k = grp; k - grp < count; k += kAttnThreads / 8) {
      const bool valid = k < count;
      const int p = start + (valid ? k : 0);
      const int8_t* ql = latent_q + static_cast<size_t>(p) * lpad;
      float dot = 0.0f;
      for (int j0 = sub * 16; j0 < Lt; j0 += 128) {
        const uint4 w = __ldcg(reinterpret_cast<const uint4*>(ql + j0));
        float f[16];
        bytes_to_f32(w.x, f);
        bytes_to_f32(w.y, f + 4);
        bytes_to_f32(w.z, f + 8);
        bytes_to_f32(w.w, f + 12);
#pragma unroll
        for (int i = 0; i < 16; ++i) dot = fmaf(qa[j0 + i], f[i], dot);
      }
      float rp = 0.0f;
      const uint16_t* kr = k_rope_cache + (static_cast<size_t>(h) * max_len + p) * rpad;
      for (int r = sub; r < rope; r += 8) rp = fmaf(qr[r], h2f(__ldcg(kr + r)), rp);
      float total = fmaf(__ldcg(latent_scale + p), dot, rp);
      total += __shfl_xor_sync(kFull, total, 4);
      total += __shfl_xor_sync(kFull, total, 2);
      total += __shfl_xor_sync(kFull, total, 1);
      if (valid && sub == 0) sc[k] = total + qb;
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int k = tid; k < count; k += kAttnThreads) mx = fmaxf(mx, sc[k]);
    mx = warp_max(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
    for (int w = 1; w < kAttnThreads / 32; ++w) mx = fmaxf(mx, red[w]);
    __syncthreads();
    const float m_new = fmaxf(m_run, mx);
    const float corr = m_run == -INFINITY ? 0.0f : expf(m_run - m_new);
    float ls = 0.0f;
    for (int k = tid; k < count; k += kAttnThreads) {
      const float e = expf(sc[k] - m_new);
      sc[k] = e * __ldcg(latent_scale + start + k);
      ls += e;
    }
    ls = warp_sum(ls);
    if (lane == 0) red[warp] = ls;
    __syncthreads();
    ls = red[0];
    for (int w = 1; w < kAttnThreads / 32; ++w) ls += red[w];
    l_run = l_run * corr + ls;
#pragma unroll
    for (int i = 0; i < 16; ++i) u[i] *= corr;
    for (int k = warp; k < count; k += kAttnThreads / 32) {
      const int8_t* ql = latent_q + static_cast<size_t>(start + k) * lpad;
      const float ea = sc[k];
#pragma unroll
      for (int pc = 0; pc < 2; ++pc) {
        const int j0 = pc * 256 + lane * 8;
        if (j0 < Lt) {
          const uint2 w = __ldcg(reinterpret_cast<const uint2*>(ql + j0));
          float f[8];
          bytes_to_f32(w.x, f);
          bytes_to_f32(w.y, f + 4);
#pragma unroll
          for (int i = 0; i < 8; ++i) u[pc * 8 + i] = fmaf(ea, f[i], u[pc * 8 + i]);
        }
      }
    }
    m_run = m_new;
    __syncthreads();
  }
#pragma unroll
  for (int pc = 0; pc < 2; ++pc) {
    const int j0 = pc * 256 + lane * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (j0 + i < Lt) part[warp][j0 + i] = u[pc * 8 + i];
  }
  __syncthreads();
  for (int j = tid; j < Lt; j += kAttnThreads) {
    float v = part[0][j];
    for (int w = 1; w < kAttnThreads / 32; ++w) v += part[w][j];
    qa[j] = v;  // the weighted latent sum u
  }
  __syncthreads();
  // out[e] = W_v[h hd + e] . u / l + b_v: thread = (output e, slice of the latent in 16-input words),
  // the slices of an output in adjacent lanes, summed by shuffles
  const IvbTernary& vu = L.v_up;
  const float inv_l = 1.0f / l_run;
  const int words = (Lt + 15) >> 4;
  int slices = kAttnThreads / hd;
  slices = slices < 1 ? 1 : (slices > 32 ? 32 : slices);
  while (slices & (slices - 1)) slices &= slices - 1;  // a power of two: lanes of one output stay in a warp
  const int per = (words + slices - 1) / slices;
  for (int base = 0; base < hd * slices; base += kAttnThreads) {
    const int item = base + tid, e = item / slices, sl = item % slices;
    float acc = 0.0f;
    if (e < hd) {
      const size_t r = static_cast<size_t>(h) * hd + e;
      const unsigned* row = reinterpret_cast<const unsigned*>(vu.packed + r * vu.row_bytes);
      for (int wd = sl * per; wd < min(words, (sl + 1) * per); ++wd) {
        const unsigned w = __ldg(row + wd);
        const float sc = h2f(__ldg(vu.scales + r * vu.scale_stride + (wd >> 3)));
        float cm1[16];
        word_codes_m1(w, cm1);
        float part_sum = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (wd * 16 + i < Lt) part_sum = fmaf(cm1[i], qa[wd * 16 + i], part_sum);
        acc = fmaf(sc, part_sum, acc);
      }
    }
    for (int off = 1; off < slices; off <<= 1) acc += __shfl_xor_sync(kFull, acc, off);
    if (e < hd && sl == 0) {
      float o = acc * inv_l;
      if (vu.bias != nullptr) o += __ldg(vu.bias + static_cast<size_t>(h) * hd + e);
      y[static_cast<size_t>(t) * d + h * hd + e] = o;
    }
  }
}


// Absorbed latent attention of every head of sequence blockIdx.x on the tensor cores: one CTA per
// sequence, 16 warps, the heads as the 16 MMA rows (heads beyond H are zero rows). Per tile of 64 cached
// positions (copied into shared memory once for all heads, cp.async, double buffered):
//   S[h][p] = <qa_h, ql_p>   (M 16 heads, N 64 positions, K latent)
//   U[h][:] = corr_h U[h][:] + sum_p w[h][p] ql_p   (M 16 heads, N latent, K 64 positions)
// with mma.sync m16n8k8 tf32: the latent codes are exact in tf32, and each fp32 operand (qa, w) is split
// into tf32 hi + lo (two MMAs), so the products keep ~21 significant bits. Between the two, warp h runs
// head h's online softmax: s_p = a_p S[h][p] + q_nope.b_k + <q_rope, k_rope_p>, w = exp(s - m) a_p.
// Then out[e] = W_v[h hd + e] . U[h] / l_h + b_v with lanes over e. Same formulas as the per-head kernel.
constexpr int kSeqWarps = 16;
constexpr int kSeqTile = 64;
constexpr int kSeqMaxNb = 4;  // latent n-blocks of 8 per warp: Lt <= 512

__device__ __forceinline__ uint32_t tf32_bits(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ void mma_tf32(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// an int8 code as the tf32 (= fp32) bits of its exact value
__device__ __forceinline__ uint32_t code_tf32(int8_t v) { return __float_as_uint(static_cast<float>(v)); }

struct SeqSmem {
  int ldq;  // floats per row of qa / u (Lp + 4)
  size_t qa_hl, qr, qb, tiles, lsc, s_part, w_hl, corr, l, u, total;
};
__host__ __device__ inline SeqSmem seq_smem(int Lp, int rope) {
  SeqSmem m;
  m.ldq = Lp + 4;
  const int lstr = Lp + 16;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += (bytes + 15) / 16 * 16;
    return at;
  };
  m.qa_hl = take(static_cast<size_t>(16) * m.ldq * 8);
  m.qr = take(static_cast<size_t>(16) * rope * 4);
  m.qb = take(16 * 4);
  m.tiles = take(static_cast<size_t>(2) * kSeqTile * lstr);
  m.lsc = take(2 * kSeqTile * 4);
  m.s_part = take(static_cast<size_t>(2) * 16 * (kSeqTile + 4) * 4);
  m.w_hl = take(static_cast<size_t>(16) * (kSeqTile + 4) * 8);
  m.corr = take(16 * 4);
  m.l = take(16 * 4);
  m.u = take(static_cast<size_t>(16) * m.ldq * 4);
  m.total = o;
  return m;
}

__global__ void __launch_bounds__(32 * kSeqWarps) batch_attention_seq_kernel(IvbLayerDesc L, IvbBatchLayer B, const float* ent,
                                                                            int ld, const int64_t* positions, int d, int Lt,
                                                                            int H, int hd, int rope, int nope, int max_len,
                                                                            int lpad, int rpad, float* y) {
  extern __shared__ __align__(16) unsigned char att_smem[];
  const int b = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;  // MMA fragment coordinates
  const int Lp = lpad;                    // latent rows padded to 16 (the pad codes are zero)
  const int lstr = Lp + 16;               // padded tile row
  const SeqSmem M = seq_smem(Lp, rope);
  const int lq = M.ldq;
  // tf32 (hi, lo) pairs, one 8-byte load per fragment element pair; the row strides (lq, kSt pairs,
  // both 4 mod 16) keep the fragment loads of a half-warp on distinct banks
  float2* qa_hl = reinterpret_cast<float2*>(att_smem + M.qa_hl);  // [16][lq] absorbed queries
  float* qr_s = reinterpret_cast<float*>(att_smem + M.qr);      // [16][rope]
  float* qb_s = reinterpret_cast<float*>(att_smem + M.qb);      // [16]
  int8_t* lat_s = reinterpret_cast<int8_t*>(att_smem + M.tiles);  // [2][kSeqTile][lstr]
  float* lsc_s = reinterpret_cast<float*>(att_smem + M.lsc);      // [2][kSeqTile]
  float* s_part = reinterpret_cast<float*>(att_smem + M.s_part);  // [2][16][kSeqTile + 4] (two K halves)
  float2* w_hl = reinterpret_cast<float2*>(att_smem + M.w_hl);    // [16][kSeqTile + 4] softmax weights
  float* corr_s = reinterpret_cast<float*>(att_smem + M.corr);    // [16]
  float* l_s = reinterpret_cast<float*>(att_smem + M.l);          // [16]
  float* u_s = reinterpret_cast<float*>(att_smem + M.u);          // [16][lq]
  constexpr int kSt = kSeqTile + 4;
  const long long pos_in = positions[b];
  if (pos_in < 0 || pos_in >= max_len) {  // capacity error, reported by the cache append
    for (int i = tid; i < H * hd; i += blockDim.x) y[static_cast<size_t>(b) * d + i] = 0.0f;
    return;
  }
  const int pos = static_cast<int>(pos_in), P = pos + 1;
  const int8_t* latent_q = B.latent_q + static_cast<size_t>(b) * max_len * lpad;
  const float* latent_scale = B.latent_scale + static_cast<size_t>(b) * max_len;
  const uint16_t* k_rope_cache = B.k_rope_cache + static_cast<size_t>(b) * H * max_len * rpad;
  const int n_tiles = (P + kSeqTile - 1) / kSeqTile;
  auto load_tile = [&](int ti) {
    const int p0 = ti * kSeqTile, cnt = min(kSeqTile, P - p0);
    int8_t* dst = lat_s + (ti & 1) * kSeqTile * lstr;
    const int chunks = Lp >> 4;  // 16-byte pieces per row
    for (int i = tid; i < cnt * chunks; i += blockDim.x) {
      const int r = i / chunks, c = i - r * chunks;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst + r * lstr + 16 * c)),
                   "l"(latent_q + static_cast<size_t>(p0 + r) * lpad + 16 * c)
                   : "memory");
    }
    for (int i = tid; i < cnt; i += blockDim.x)
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(lsc_s + (ti & 1) * kSeqTile + i)),
                   "l"(latent_scale + p0 + i)
                   : "memory");
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  load_tile(0);
  // rows of heads >= H stay zero: no score, no weight
  for (int i = tid; i < 16 * kSt; i += blockDim.x) {
    w_hl[i] = make_float2(0.0f, 0.0f);
  }
  // absorbed queries (tf32 hi/lo), rotated rope queries and q_nope . b_k of every head (warp per head);
  // lane = (e slice, 16-input word): slices of the nope inputs meet by shuffles
  const float scl = L.attn_scale;
  const float* rtab = L.rope + static_cast<size_t>(pos) * rope;
  const IvbTernary& kn = L.k_nope_up;
  const int words = Lp >> 4;
  const int slices = words >= 32 ? 1 : 32 / words;  // words is a power of two <= 32 (Lp <= 512)
  // the queries of all heads into shared memory (the u rows are free until the end)
  for (int i = tid; i < H * hd; i += blockDim.x) u_s[i] = ent[static_cast<size_t>(b) * ld + i];
  __syncthreads();
  {
    const int h = warp;
    const bool live = h < H;
    const float* q = u_s + h * hd;
    if (live)
      for (int jr = lane; jr < rope / 2; jr += 32) {
        const float cs = __ldg(rtab + 2 * jr), sn = __ldg(rtab + 2 * jr + 1);
        const float q0 = q[nope + 2 * jr], q1 = q[nope + 2 * jr + 1];
        qr_s[h * rope + 2 * jr] = (q0 * cs - q1 * sn) * scl;
        qr_s[h * rope + 2 * jr + 1] = (q0 * sn + q1 * cs) * scl;
      }
    const int wd = lane % words, sl = lane / words;
    float acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.0f;
    if (live && sl < slices) {
#pragma unroll 8
      for (int e = sl; e < nope; e += slices) {
        const size_t r = static_cast<size_t>(h) * nope + e;
        const unsigned w = __ldg(reinterpret_cast<const unsigned*>(kn.packed + r * kn.row_bytes) + wd);
        const float qs = q[e] * scl * h2f(__ldg(kn.scales + r * kn.scale_stride + (wd >> 3)));
        float cm1[16];
        word_codes_m1(w, cm1);
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = fmaf(qs, cm1[i], acc[i]);
      }
    }
    for (int off = words; off < 32; off <<= 1)
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] += __shfl_xor_sync(kFull, acc[i], off);
    if (sl == 0)
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float v = live ? acc[i] : 0.0f;
        const uint32_t hi = tf32_bits(v);
        qa_hl[h * lq + wd * 16 + i] = make_float2(__uint_as_float(hi), __uint_as_float(tf32_bits(v - __uint_as_float(hi))));
      }
    float pp = 0.0f;
    if (live && kn.bias != nullptr)
      for (int e = lane; e < nope; e += 32) pp = fmaf(q[e] * scl, __ldg(kn.bias + h * nope + e), pp);
    pp = warp_sum(pp);
    if (lane == 0) qb_s[h] = pp;
  }
  // head h's softmax state (warp h); U accumulators of latent n-blocks warp, warp + 16, ...
  float m_run = -INFINITY, l_run = 0.0f;
  float uacc[kSeqMaxNb][4];
#pragma unroll
  for (int j = 0; j < kSeqMaxNb; ++j)
#pragma unroll
    for (int c = 0; c < 4; ++c) uacc[j][c] = 0.0f;
  const int ksteps = Lp >> 3, khalf = (ksteps + 1) >> 1;
  for (int ti = 0; ti < n_tiles; ++ti) {
    __syncthreads();  // the previous tile's buffer, scores and weights are no longer read
    if (ti + 1 < n_tiles) {
      load_tile(ti + 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const int p0 = ti * kSeqTile, cnt = min(kSeqTile, P - p0);
    const int8_t* tile = lat_s + (ti & 1) * kSeqTile * lstr;
    const float* lsc = lsc_s + (ti & 1) * kSeqTile;
    // head warp's rotated keys of its two positions, issued together before the score MMAs (rpad <= 32:
    // up to four 16-byte loads per position), so their latency is paid once and hidden
    constexpr int kKrVec = 4;
    uint4 krv[2][kKrVec];
    const bool kr_vec = rpad <= 8 * kKrVec;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int pl = lane + 32 * k;
      const uint4* kr4 = reinterpret_cast<const uint4*>(k_rope_cache + (static_cast<size_t>(warp) * max_len + p0 + pl) * rpad);
      const bool ok = kr_vec && warp < H && pl < cnt;
#pragma unroll
      for (int v = 0; v < kKrVec; ++v) krv[k][v] = ok && 8 * v < rpad ? __ldg(kr4 + v) : make_uint4(0u, 0u, 0u, 0u);
    }
    // ---- S = QA x tile^T: warp -> positions 8 (warp % 8).., K half warp / 8 ----
    {
      const int nb = warp & 7, half = warp >> 3;
      const int k_lo = half * khalf, k_hi = min(ksteps, k_lo + khalf);
      float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      const int8_t* prow = tile + (8 * nb + g) * lstr;
      for (int ks = k_lo; ks < k_hi; ++ks) {
        const int k0 = 8 * ks;
        const uint32_t b0 = code_tf32(prow[k0 + t]), b1 = code_tf32(prow[k0 + t + 4]);
        const float2 a0 = qa_hl[g * lq + k0 + t], a1 = qa_hl[(g + 8) * lq + k0 + t];
        const float2 a2 = qa_hl[g * lq + k0 + t + 4], a3 = qa_hl[(g + 8) * lq + k0 + t + 4];
        mma_tf32(c, __float_as_uint(a0.x), __float_as_uint(a1.x), __float_as_uint(a2.x), __float_as_uint(a3.x), b0, b1);
        mma_tf32(c, __float_as_uint(a0.y), __float_as_uint(a1.y), __float_as_uint(a2.y), __float_as_uint(a3.y), b0, b1);
      }
      float* sp = s_part + half * 16 * kSt;
      sp[g * kSt + 8 * nb + 2 * t] = c[0];
      sp[g * kSt + 8 * nb + 2 * t + 1] = c[1];
      sp[(g + 8) * kSt + 8 * nb + 2 * t] = c[2];
      sp[(g + 8) * kSt + 8 * nb + 2 * t + 1] = c[3];
    }
    __syncthreads();
    // ---- online softmax of head h = warp over the tile's positions ----
    if (warp < H) {
      const int h = warp;
      const float qb = qb_s[h];
      float s2[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int pl = lane + 32 * k;
        s2[k] = -INFINITY;
        if (pl < cnt) {
          const float dot = s_part[h * kSt + pl] + s_part[16 * kSt + h * kSt + pl];
          float rp = 0.0f;
          if (kr_vec) {
#pragma unroll
            for (int v = 0; v < kKrVec; ++v) {
              const uint32_t kw[4] = {krv[k][v].x, krv[k][v].y, krv[k][v].z, krv[k][v].w};  // halves 8v .. 8v + 7
#pragma unroll
              for (int r2 = 0; r2 < 8; ++r2) {
                const int r = 8 * v + r2;
                if (r < rope) rp = fmaf(qr_s[h * rope + r], h2f(static_cast<uint16_t>(kw[r2 >> 1] >> (16 * (r2 & 1)))), rp);
              }
            }
          } else {
            const uint16_t* kr = k_rope_cache + (static_cast<size_t>(h) * max_len + p0 + pl) * rpad;
            for (int r = 0; r < rope; ++r) rp = fmaf(qr_s[h * rope + r], h2f(__ldg(kr + r)), rp);
          }
          s2[k] = fmaf(lsc[pl], dot, rp) + qb;
        }
      }
      const float mx = warp_max(fmaxf(s2[0], s2[1]));
      const float m_new = fmaxf(m_run, mx);
      const float corr = m_run == -INFINITY ? 0.0f : expf(m_run - m_new);
      float ls = 0.0f;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int pl = lane + 32 * k;
        float wgt = 0.0f;
        if (pl < cnt) {
          const float e = expf(s2[k] - m_new);
          ls += e;
          wgt = e * lsc[pl];
        }
        const uint32_t hi = tf32_bits(wgt);
        w_hl[h * kSt + pl] = make_float2(__uint_as_float(hi), __uint_as_float(tf32_bits(wgt - __uint_as_float(hi))));
      }
      ls = warp_sum(ls);
      l_run = l_run * corr + ls;
      m_run = m_new;
      if (lane == 0) corr_s[h] = corr;
    } else if (warp < 16 && lane == 0) {
      corr_s[warp] = 1.0f;
    }
    __syncthreads();
    // ---- U = corr U + W x tile: warp -> latent n-blocks warp, warp + 16, ... ----
    {
      const float c_lo = corr_s[g], c_hi = corr_s[g + 8];
      const int nbs = Lp >> 3;
#pragma unroll
      for (int j = 0; j < kSeqMaxNb; ++j) {
        const int nb = warp + 16 * j;
        if (nb < nbs) {
          uacc[j][0] *= c_lo;
          uacc[j][1] *= c_lo;
          uacc[j][2] *= c_hi;
          uacc[j][3] *= c_hi;
#pragma unroll
          for (int ks = 0; ks < kSeqTile / 8; ++ks) {
            const int k0 = 8 * ks;
            const uint32_t b0 = code_tf32(tile[(k0 + t) * lstr + 8 * nb + g]);
            const uint32_t b1 = code_tf32(tile[(k0 + t + 4) * lstr + 8 * nb + g]);
            const float2 a0 = w_hl[g * kSt + k0 + t], a1 = w_hl[(g + 8) * kSt + k0 + t];
            const float2 a2 = w_hl[g * kSt + k0 + t + 4], a3 = w_hl[(g + 8) * kSt + k0 + t + 4];
            mma_tf32(uacc[j], __float_as_uint(a0.x), __float_as_uint(a1.x), __float_as_uint(a2.x), __float_as_uint(a3.x), b0, b1);
            mma_tf32(uacc[j], __float_as_uint(a0.y), __float_as_uint(a1.y), __float_as_uint(a2.y), __float_as_uint(a3.y), b0, b1);
          }
        }
      }
    }
  }
  if (warp < H && lane == 0) l_s[warp] = l_run;
  __syncthreads();
  {
    const int nbs = Lp >> 3;
    const float il_lo = g < H ? 1.0f / l_s[g] : 0.0f, il_hi = g + 8 < H ? 1.0f / l_s[g + 8] : 0.0f;
#pragma unroll
    for (int j = 0; j < kSeqMaxNb; ++j) {
      const int nb = warp + 16 * j;
      if (nb < nbs) {
        u_s[g * lq + 8 * nb + 2 * t] = uacc[j][0] * il_lo;
        u_s[g * lq + 8 * nb + 2 * t + 1] = uacc[j][1] * il_lo;
        u_s[(g + 8) * lq + 8 * nb + 2 * t] = uacc[j][2] * il_hi;
        u_s[(g + 8) * lq + 8 * nb + 2 * t + 1] = uacc[j][3] * il_hi;
      }
    }
  }
  __syncthreads();
  // out = W_v u / l + b_v: warp per head, lanes over the outputs e
  if (warp < H) {
    const int h = warp;
    const float* us = u_s + h * lq;
    const IvbTernary& vu = L.v_up;
    for (int e = lane; e < hd; e += 32) {
      const size_t r = static_cast<size_t>(h) * hd + e;
      const unsigned* row = reinterpret_cast<const unsigned*>(vu.packed + r * vu.row_bytes);
      float acc = 0.0f;
#pragma unroll 8
      for (int wd = 0; wd < words; ++wd) {
        const unsigned w = __ldg(row + wd);
        float cm1[16], uv[16];
        word_codes_m1(w, cm1);
#pragma unroll
        for (int i = 0; i < 4; ++i) *reinterpret_cast<float4*>(uv + 4 * i) = reinterpret_cast<const float4*>(us + wd * 16)[i];
        float part_sum = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) part_sum = fmaf(cm1[i], uv[i], part_sum);
        acc = fmaf(h2f(__ldg(vu.scales + r * vu.scale_stride + (wd >> 3))), part_sum, acc);
      }
      if (vu.bias != nullptr) acc += __ldg(vu.bias + r);
      y[static_cast<size_t>(b) * d + h * hd + e] = acc;
    }
  }
}

// Sampler of sequence blockIdx.x (temperature, repetition penalty, top-k, Philox draw), then its
// position advances by one.
__global__ void __launch_bounds__(kThreads, 1) batch_sample_kernel(const float* logits, uint8_t* seen, int vocab,
                                                                   const float* sampling, const int64_t* top_k,
                                                                   int max_top_k, uint64_t* rng, int64_t* tokens,
                                                                   int64_t* positions, int64_t* history, int history_len,
                                                                   const int32_t* step_counter) {
  extern __shared__ __align__(16) unsigned char smem[];
  SampleSmem sm;
  carve_sample(smem, vocab, sm);
  const int b = blockIdx.x;
  const int step = step_counter != nullptr ? *step_counter - 1 : -1;  // advanced by this step's embedding kernel
  int64_t* hist = (history != nullptr && step >= 0 && step < history_len) ? history + static_cast<size_t>(b) * history_len + step
                                                                         : nullptr;
  sample_block(logits + static_cast<size_t>(b) * vocab, seen + static_cast<size_t>(b) * vocab, vocab, sampling, top_k,
               max_top_k, rng + 2 * b, tokens + b, hist, sm);
  if (threadIdx.x == 0) positions[b] += 1;
}

// ---- vocabulary-sharded sampling (tensor parallel) ----------------------------------------------
// The requested top-k as every sampler clamps it.
__device__ __forceinline__ int sampler_k(const int64_t* top_k, int max_top_k, int vocab) {
  const long long kreq = ldcg_i64(top_k);
  const int cap = min(min(max_top_k, vocab), kMaxTopK);
  return static_cast<int>(kreq < 1 ? 1 : (kreq > cap ? cap : kreq));
}

// Sequence blockIdx.x, one rank's vocabulary slice [v0, v0 + vloc): the scores of its logits and
// repetition flags (the sampler's keys), their top min(K, vloc) by (key desc, index asc) into slots
// [0, kc) of keys / ids (global ids), the rest padded with key 0, below every score.
__global__ void __launch_bounds__(kThreads, 1) batch_topk_slice_kernel(const float* logits, const uint8_t* seen, int vloc, int v0,
                                                                       int vocab, const float* sampling, const int64_t* top_k,
                                                                       int max_top_k, int kc, unsigned* keys, int* ids) {
  extern __shared__ __align__(16) unsigned char smem[];
  SampleSmem sm;
  carve_sample(smem, vloc, sm);
  const int b = blockIdx.x, tid = threadIdx.x;
  const float* lg = logits + static_cast<size_t>(b) * vloc;
  const uint8_t* fl = seen + static_cast<size_t>(b) * vloc;
  const float inv_t = 1.0f / __ldcg(sampling);
  const float pen = __ldcg(sampling + 1), ipen = __ldcg(sampling + 2);
  for (int i = tid; i < vloc; i += kThreads) sm.keys[i] = score_key(__ldcg(lg + i), __ldcg(fl + i), inv_t, pen, ipen);
  __syncthreads();
  const int kl = min(sampler_k(top_k, max_top_k, vocab), vloc);
  select_topk(sm, vloc, kl);
  for (int r = tid; r < kc; r += kThreads) {
    keys[static_cast<size_t>(b) * kc + r] = r < kl ? sm.hist[r] : 0u;
    ids[static_cast<size_t>(b) * kc + r] = r < kl ? v0 + static_cast<int>(sm.hist[kMaxTopK + r]) : vocab + r;
  }
}

// Sequence blockIdx.x: the candidates of all ranks ([world][batch][kc], rank-major, each rank's list in
// (key desc, id asc) order, so the position order of equal keys is their id order) merged by the same
// selection and draw as the unsharded sampler, which therefore picks the same token; then history,
// position, and the repetition flag when the token lies in this rank's slice [v0, v0 + vloc).
__global__ void __launch_bounds__(kThreads, 1) batch_merge_sample_kernel(const unsigned* keys, const int* ids, int world, int batch,
                                                                         int kc, int vocab, const int64_t* top_k, int max_top_k,
                                                                         uint64_t* rng, int64_t* tokens, int64_t* positions,
                                                                         int64_t* history, int history_len,
                                                                         const int32_t* step_counter, uint8_t* seen, int v0,
                                                                         int vloc) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int n = world * kc;
  SampleSmem sm;
  carve_sample(smem, n, sm);
  int* cid = reinterpret_cast<int*>(smem + sample_smem_bytes(n));
  const int b = blockIdx.x, tid = threadIdx.x;
  for (int i = tid; i < n; i += kThreads) {
    const int r = i / kc, j = i - r * kc;
    const size_t src = (static_cast<size_t>(r) * batch + b) * kc + j;
    sm.keys[i] = keys[src];
    cid[i] = ids[src];
  }
  __syncthreads();
  const int K = sampler_k(top_k, max_top_k, vocab);
  select_topk(sm, n, K);
  const int chosen = draw_sorted(sm, K, rng + 2 * b);
  if (tid == 0) {
    const int token = cid[sm.hist[kMaxTopK + chosen]];
    tokens[b] = token;
    const int step = step_counter != nullptr ? *step_counter - 1 : -1;  // advanced by this step's embedding kernel
    if (history != nullptr && step >= 0 && step < history_len) history[static_cast<size_t>(b) * history_len + step] = token;
    if (token >= v0 && token < v0 + vloc) seen[static_cast<size_t>(b) * vloc + (token - v0)] = 1;
    positions[b] += 1;
  }
}

// One CTA per sequence (a warp per head, the latent tiles shared) when there are enough sequences to fill
// the SMs and the heads fit in one CTA; else one CTA per (sequence, head), more parallel for few sequences.
int32_t launch_batch_attention(const IvbLayerDesc& L, const IvbBatchLayer& BL, const float* ent, int ld, const int64_t* positions,
                               int batch, int d, int Lt, int H, int hd, int rope, int nope, int max_len, int lpad, int rpad,
                               float* y, cudaStream_t s) {
  const int words = lpad / 16;
  if (H <= kSeqWarps && Lt <= 512 && (words & (words - 1)) == 0 && batch >= 128) {
    const size_t smem = seq_smem(lpad, rope).total;
    IVB_CUDA(cudaFuncSetAttribute(batch_attention_seq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    batch_attention_seq_kernel<<<batch, 32 * kSeqWarps, smem, s>>>(L, BL, ent, ld, positions, d, Lt, H, hd, rope, nope, max_len,
                                                                   lpad, rpad, y);
  } else {
    batch_attention_kernel<<<dim3(batch, H), kAttnThreads, 0, s>>>(L, BL, ent, ld, positions, d, Lt, H, hd, rope, nope, max_len,
                                                                   lpad, rpad, y);
  }
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

struct BatchLayout {
  size_t resid, ent, y, h, q8, scale, partial, total;
  int ldq;
};

BatchLayout batch_layout(const IvbModelDesc& md, const IvbLayerDesc* layers, int batch) {
  BatchLayout L{};
  const int d = md.hidden, F = md.dense;
  int ld_ent = 0;
  for (int i = 0; i < md.num_layers; ++i) ld_ent = std::max(ld_ent, layers[i].entry.rows);
  L.ldq = (std::max(d, F) + 127) / 128 * 128;
  const size_t T = static_cast<size_t>(batch);
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  L.resid = take(T * d * 4);
  L.ent = take(T * ld_ent * 4);
  L.y = take(T * d * 4);
  L.h = take(T * std::max(F, d) * 4);
  L.q8 = take((T + 127) / 128 * 128 * L.ldq);
  L.scale = take(T * 4);
  L.partial = take(kGemmPartialFloats * 4);  // split-K partial sums of this call's GEMMs
  L.total = o;
  return L;
}

}  // namespace
}  // namespace ivb

extern "C" {

uint64_t ivb_batch_workspace_bytes(const IvbDecoder* dec, int32_t batch) {
  using namespace ivb;
  if (dec == nullptr || batch <= 0) return 0;
  const IvbLayerDesc* layers = nullptr;
  const IvbModelDesc& md = decoder_model(dec, &layers);
  return batch_layout(md, layers, batch).total;
}

int32_t ivb_batch_decode(IvbDecoder* dec, const IvbBatch* bt, int32_t steps, void* workspace, uint64_t workspace_bytes,
                         void* stream) {
  using namespace ivb;
  if (dec == nullptr || bt == nullptr || workspace == nullptr) return fail(IVB_EINVAL, "ivb_batch_decode: null argument");
  if (bt->layers == nullptr || bt->tokens == nullptr || bt->positions == nullptr || bt->logits == nullptr ||
      bt->seen == nullptr || bt->rng == nullptr || bt->sampling == nullptr || bt->top_k == nullptr)
    return fail(IVB_EINVAL, "ivb_batch_decode: null batch buffer");
  const int B = bt->batch;
  if (B <= 0 || steps < 0) return fail(IVB_EINVAL, "ivb_batch_decode: batch %d, steps %d", B, steps);
  const IvbLayerDesc* layers = nullptr;
  const IvbModelDesc& md = decoder_model(dec, &layers);
  const BatchLayout W = batch_layout(md, layers, B);
  if (workspace_bytes < W.total) return fail(IVB_EINVAL, "ivb_batch_decode: workspace too small (%llu < %zu)",
                                             static_cast<unsigned long long>(workspace_bytes), W.total);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return fail(IVB_EINVAL, "ivb_batch_decode: workspace must be 256-byte aligned");
  const int d = md.hidden, F = md.dense, H = md.heads, hd = md.head_dim, S = md.state_dim, Lt = md.latent_dim;
  const int rope = md.rope_dim, nope = md.nope_dim, V = md.vocab;
  if (Lt > 512 || rope > 128 || nope > 256 || S > 16) return fail(IVB_EINVAL, "ivb_batch_decode: shapes beyond the batch kernels");
  for (int i = 0; i < md.num_layers; ++i)
    if (layers[i].kind == IVB_MAMBA && layers[i].conv_taps > kBatchTaps + 1)
      return fail(IVB_EINVAL, "ivb_batch_decode: conv width %d beyond the step kernel", layers[i].conv_taps);
  uint32_t* err = decoder_error_word(dec);
  if (err == nullptr) return fail(IVB_EINVAL, "ivb_batch_decode: bind the decoder first");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  float* resid = reinterpret_cast<float*>(ws + W.resid);
  float* ent = reinterpret_cast<float*>(ws + W.ent);
  float* y = reinterpret_cast<float*>(ws + W.y);
  float* hbuf = reinterpret_cast<float*>(ws + W.h);
  int8_t* q8 = reinterpret_cast<int8_t*>(ws + W.q8);
  float* scale = reinterpret_cast<float*>(ws + W.scale);
  const int lpad = (Lt + 15) / 16 * 16, rpad = (rope + 7) / 8 * 8;
  const size_t sample_smem = sample_smem_bytes(V);
  IVB_CUDA(cudaFuncSetAttribute(batch_sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sample_smem)));
  auto quant = [&](const float* x, int n, const float* norm, float eps) -> int32_t {
    const int ld = (n + 127) / 128 * 128;
    return ivb_quantize_rows(x, B, n, norm, eps, md.norm_clip, md.act_eps, q8, ld, scale, nullptr, stream);
  };
  float* partial = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + W.partial);
  auto gemm = [&](const IvbTernary& m, int epilogue, float* out, int ldo) -> int32_t {
    const int ld = (m.in_features + 127) / 128 * 128;
    return ternary_gemm_into(&m, q8, ld, scale, B, epilogue, out, ldo, err, partial, kGemmPartialFloats, stream);
  };
  for (int step = 0; step < steps; ++step) {
    batch_embed_kernel<<<B, kThreads, 0, s>>>(md.head, bt->tokens, d, resid, bt->step);
    IVB_CUDA(cudaGetLastError());
    for (int li = 0; li < md.num_layers; ++li) {
      const IvbLayerDesc& L = layers[li];
      const IvbBatchLayer& BL = bt->layers[li];
      const int ld = L.entry.rows;
      if (int32_t rc = quant(resid, d, L.mixer_norm, L.mixer_norm_eps)) return rc;
      if (int32_t rc = gemm(L.entry, IVB_EPI_STORE, ent, ld)) return rc;
      if (L.kind == IVB_MAMBA) {
        const int nh_max = std::min(H, kSsmChannels / hd + 2);
        batch_ssm_kernel<<<dim3((d + kSsmChannels - 1) / kSsmChannels, B), kSsmChannels, nh_max * S * 5 * 4, s>>>(
            L, BL, ent, ld, d, H, hd, S, L.conv_taps, L.half_dt_min, L.half_dt_range, y);
        IVB_CUDA(cudaGetLastError());
      } else {
        batch_cache_kernel<<<B, kThreads, 0, s>>>(L, BL, ent, ld, bt->positions, d, Lt, H, rope, md.max_len, lpad, rpad,
                                                  md.act_eps, err);
        IVB_CUDA(cudaGetLastError());
        if (int32_t rc = launch_batch_attention(L, BL, ent, ld, bt->positions, B, d, Lt, H, hd, rope, nope, md.max_len, lpad,
                                                rpad, y, s))
          return rc;
      }
      if (int32_t rc = quant(y, d, nullptr, 0.0f)) return rc;
      if (int32_t rc = gemm(L.out, IVB_EPI_RESIDUAL, resid, d)) return rc;
      if (int32_t rc = quant(resid, d, L.ffn_norm, L.ffn_norm_eps)) return rc;
      if (int32_t rc = gemm(L.gate_up, IVB_EPI_SILU_PAIR, hbuf, F)) return rc;
      if (int32_t rc = quant(hbuf, F, nullptr, 0.0f)) return rc;
      if (int32_t rc = gemm(L.down, IVB_EPI_RESIDUAL, resid, d)) return rc;
    }
    if (int32_t rc = quant(resid, d, md.final_norm, md.final_norm_eps)) return rc;
    if (int32_t rc = gemm(md.head, IVB_EPI_STORE, bt->logits, V)) return rc;
    batch_sample_kernel<<<B, kThreads, sample_smem, s>>>(bt->logits, bt->seen, V, bt->sampling, bt->top_k, md.max_top_k,
                                                         bt->rng, bt->tokens, bt->positions, bt->history, bt->history_len,
                                                         bt->step);
    IVB_CUDA(cudaGetLastError());
  }
  return IVB_OK;
}

// ---- unit steps, for callers that orchestrate the layers themselves (tensor parallel) -----------

int32_t ivb_batch_embed(const IvbTernary* head, const int64_t* tokens, int32_t batch, int32_t hidden, float* resid,
                        int32_t* step_counter, void* stream) {
  using namespace ivb;
  if (head == nullptr || tokens == nullptr || resid == nullptr || batch <= 0 || hidden <= 0)
    return fail(IVB_EINVAL, "ivb_batch_embed: bad argument");
  batch_embed_kernel<<<batch, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(*head, tokens, hidden, resid, step_counter);
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

int32_t ivb_batch_ssm(const IvbLayerDesc* L, const IvbBatchLayer* B, const float* ent, int32_t ld, int32_t batch,
                      int32_t channels, int32_t heads, int32_t head_dim, int32_t state_dim, float* y, void* stream) {
  using namespace ivb;
  if (L == nullptr || B == nullptr || ent == nullptr || y == nullptr || batch <= 0 || channels != heads * head_dim ||
      state_dim > 16 || L->conv_taps > kBatchTaps + 1)
    return fail(IVB_EINVAL, "ivb_batch_ssm: bad argument");
  const int nh_max = std::min(heads, kSsmChannels / head_dim + 2);
  batch_ssm_kernel<<<dim3((channels + kSsmChannels - 1) / kSsmChannels, batch), kSsmChannels,
                     nh_max * state_dim * 5 * 4, static_cast<cudaStream_t>(stream)>>>(
      *L, *B, ent, ld, channels, heads, head_dim, state_dim, L->conv_taps, L->half_dt_min, L->half_dt_range, y);
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

int32_t ivb_batch_mla(const IvbLayerDesc* L, const IvbBatchLayer* B, const float* ent, int32_t ld, const int64_t* positions,
                      int32_t batch, int32_t channels, int32_t latent, int32_t heads, int32_t head_dim, int32_t rope,
                      int32_t nope, int32_t max_len, float act_eps, uint32_t* error, float* y, void* stream) {
  using namespace ivb;
  if (L == nullptr || B == nullptr || ent == nullptr || positions == nullptr || y == nullptr || error == nullptr ||
      batch <= 0 || channels != heads * head_dim || latent > 512 || rope > 128 || nope > 256)
    return fail(IVB_EINVAL, "ivb_batch_mla: bad argument");
  const int lpad = (latent + 15) / 16 * 16, rpad = (rope + 7) / 8 * 8;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  batch_cache_kernel<<<batch, kThreads, 0, s>>>(*L, *B, ent, ld, positions, channels, latent, heads, rope, max_len, lpad, rpad,
                                                act_eps, error);
  IVB_CUDA(cudaGetLastError());
  if (int32_t rc = launch_batch_attention(*L, *B, ent, ld, positions, batch, channels, latent, heads, head_dim, rope, nope,
                                          max_len, lpad, rpad, y, s))
    return rc;
  return IVB_OK;
}

int32_t ivb_batch_sample(const float* logits, uint8_t* seen, int32_t vocab, int32_t batch, const float* sampling,
                         const int64_t* top_k, int32_t max_top_k, uint64_t* rng, int64_t* tokens, int64_t* positions,
                         int64_t* history, int32_t history_len, const int32_t* step_counter, void* stream) {
  using namespace ivb;
  if (logits == nullptr || seen == nullptr || sampling == nullptr || top_k == nullptr || rng == nullptr ||
      tokens == nullptr || positions == nullptr || batch <= 0 || vocab <= 0)
    return fail(IVB_EINVAL, "ivb_batch_sample: bad argument");
  const size_t smem = sample_smem_bytes(vocab);
  IVB_CUDA(cudaFuncSetAttribute(batch_sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  batch_sample_kernel<<<batch, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      logits, seen, vocab, sampling, top_k, max_top_k, rng, tokens, positions, history, history_len, step_counter);
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

int32_t ivb_batch_topk_slice(const float* logits, const uint8_t* seen, int32_t vloc, int32_t v0, int32_t vocab, int32_t batch,
                             const float* sampling, const int64_t* top_k, int32_t max_top_k, int32_t kc, uint32_t* keys,
                             int32_t* ids, void* stream) {
  using namespace ivb;
  if (logits == nullptr || seen == nullptr || sampling == nullptr || top_k == nullptr || keys == nullptr || ids == nullptr ||
      batch <= 0 || vloc <= 0 || v0 < 0 || v0 + vloc > vocab || kc < std::min(std::min(max_top_k, vocab), kMaxTopK) || kc <= 0)
    return fail(IVB_EINVAL, "ivb_batch_topk_slice: bad argument");
  const size_t smem = sample_smem_bytes(vloc);
  IVB_CUDA(cudaFuncSetAttribute(batch_topk_slice_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  batch_topk_slice_kernel<<<batch, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(logits, seen, vloc, v0, vocab, sampling,
                                                                                         top_k, max_top_k, kc, keys, ids);
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

int32_t ivb_batch_sample_merge(const uint32_t* keys, const int32_t* ids, int32_t world, int32_t batch, int32_t kc, int32_t vocab,
                               const int64_t* top_k, int32_t max_top_k, uint64_t* rng, int64_t* tokens, int64_t* positions,
                               int64_t* history, int32_t history_len, const int32_t* step_counter, uint8_t* seen, int32_t v0,
                               int32_t vloc, void* stream) {
  using namespace ivb;
  if (keys == nullptr || ids == nullptr || top_k == nullptr || rng == nullptr || tokens == nullptr || positions == nullptr ||
      seen == nullptr || world <= 0 || batch <= 0 || kc <= 0 || vocab <= 0 || vloc <= 0 || v0 < 0 || v0 + vloc > vocab)
    return fail(IVB_EINVAL, "ivb_batch_sample_merge: bad argument");
  const size_t smem = sample_smem_bytes(world * kc) + static_cast<size_t>(world) * kc * 4;
  IVB_CUDA(cudaFuncSetAttribute(batch_merge_sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  batch_merge_sample_kernel<<<batch, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      keys, ids, world, batch, kc, vocab, top_k, max_top_k, rng, tokens, positions, history, history_len, step_counter, seen, v0,
      vloc);
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

}  // extern "C"
