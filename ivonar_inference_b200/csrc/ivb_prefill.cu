// Prompt prefill of libivonar_b200.so: all prompt tokens of a chunk go through each layer together.
//
// Per block: quantise every token row (ivb_quantize_rows), the entry projection as one tcgen05 int8
// GEMM over all tokens (ivb_ternary_gemm), then the mixer — the recurrent scan over the tokens for a
// mamba block (one warp lane per state, tokens in order), or for an mla block the latent/k_rope cache
// fill of every token followed by causal latent attention (one CTA per token and head) — then the
// out, gate/up and down GEMMs with their residual / SwiGLU epilogues. The head runs on the last
// token only. Caches, recurrent state, position and token end exactly where the token-by-token decode
// kernel would leave them, so decoding continues from here. Replaces kernel_decoder.py:457-479
// (prefill) and kernels/ternary.cu:688-982 (tile GEMM, recurrent tile, kv write, attention tile).
#include <cuda_runtime.h>

#include <algorithm>

#include "ivb_common.h"
#include "ivb_cluster.cuh"

namespace ivb {

const IvbModelDesc& decoder_model(const IvbDecoder* dec, const IvbLayerDesc** layers);
unsigned* decoder_error_word(const IvbDecoder* dec);

constexpr int kMaxTaps = 8;

// Embedding rows of the prompt tokens (the tied head): resid[t][i] = (code - 1) * scale.
__global__ void __launch_bounds__(kThreads) embed_rows_kernel(IvbTernary head, const int64_t* tokens, int d, float* resid) {
  const int t = blockIdx.x;
  const long long tok = tokens[t];
  const uint8_t* erow = head.packed + static_cast<size_t>(tok) * head.row_bytes;
  const uint16_t* srow = head.scales + static_cast<size_t>(tok) * head.scale_stride;
  for (int i = threadIdx.x; i < d; i += kThreads)
    resid[static_cast<size_t>(t) * d + i] =
        static_cast<float>(((__ldg(erow + (i >> 2)) >> ((i & 3) << 1)) & 3) - 1) * h2f(__ldg(srow + (i >> 7)));
}

// Recurrent scan of one mamba block over T tokens. ent [T][2d + 3HS]: value | gate | per head (B, C, dt).
// A half-warp per channel, lane s owns state s; tokens in order. Same arithmetic as the decode step.
__global__ void __launch_bounds__(kThreads) ssm_scan_kernel(IvbLayerDesc L, const float* ent, int T, int d, int H, int hd,
                                                            int S, int taps, float half_dt_min, float half_dt_range,
                                                            float* y) {
  const int lane = threadIdx.x & 31, sub = lane & 15;
  const int c = (blockIdx.x * kThreads + threadIdx.x) >> 4;  // channel
  const bool live = c < d;
  const int cc_ = live ? c : 0;
  const int h = cc_ / hd, dd = cc_ - h * hd;
  const int ld = 2 * d + 3 * H * S;
  const bool on = live && sub < S;
  const int s = on ? sub : 0;
  float win[kMaxTaps];
#pragma unroll
  for (int k = 0; k < kMaxTaps; ++k) win[k] = (k < taps - 1 && live) ? L.conv_state[static_cast<size_t>(cc_) * (taps - 1) + k] : 0.0f;
  const size_t si_idx = (static_cast<size_t>(h) * S + s) * hd + dd;
  float sr = on ? L.ssm_state[2 * si_idx] : 0.0f, si = on ? L.ssm_state[2 * si_idx + 1] : 0.0f;
  float prev = on ? L.prev_force[si_idx] : 0.0f;
  const float decay = on ? L.decay[h * S + s] : 0.0f, theta = on ? L.theta[h * S + s] : 0.0f;
  const float skip = live ? L.skip[cc_] : 0.0f, convb = live ? L.conv_bias[cc_] : 0.0f;
  for (int t = 0; t < T; ++t) {
    const float* row = ent + static_cast<size_t>(t) * ld;
    const float incoming = live ? row[cc_] : 0.0f;
    float conv = convb;
    for (int k2 = 0; k2 < taps - 1; ++k2) conv = fmaf(live ? L.conv_weight[cc_ * taps + k2] : 0.0f, win[k2], conv);
    conv = fmaf(live ? L.conv_weight[cc_ * taps + taps - 1] : 0.0f, incoming, conv);
#pragma unroll
    for (int k2 = 0; k2 + 1 < kMaxTaps; ++k2)
      if (k2 + 1 < taps - 1) win[k2] = win[k2 + 1];
#pragma unroll
    for (int k2 = 0; k2 < kMaxTaps; ++k2)
      if (k2 == taps - 2) win[k2] = incoming;
    const float value = silu_f(conv);
    float contrib = 0.0f;
    if (on) {
      const float* bcdt = row + 2 * d + h * 3 * S;
      const float half_dt = half_dt_min + sigmoid_f(bcdt[2 * S + s]) * half_dt_range;
      const float mag = expf(2.0f * half_dt * decay);
      float sn, cs;
      sincosf(2.0f * half_dt * theta, &sn, &cs);
      const float ar = mag * cs, ai = mag * sn;
      const float b = tanhf(bcdt[s]), cc = tanhf(bcdt[S + s]);
      const float force = b * value;
      const float dr = (force + ar * prev) * half_dt;
      const float di = (ai * prev) * half_dt;
      const float nr = sr * ar - si * ai + dr;
      const float ni = sr * ai + si * ar + di;
      sr = nr;
      si = ni;
      prev = force;
      contrib = cc * nr;
    }
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) contrib += __shfl_xor_sync(kFull, contrib, off);
    if (live && sub == 0) y[static_cast<size_t>(t) * d + cc_] = (contrib + skip * value) * sigmoid_f(row[d + cc_]);
  }
  if (on) {
    L.ssm_state[2 * si_idx] = sr;
    L.ssm_state[2 * si_idx + 1] = si;
    L.prev_force[si_idx] = prev;
  }
  if (live && sub == 0)
    for (int k = 0; k < taps - 1; ++k) L.conv_state[static_cast<size_t>(cc_) * (taps - 1) + k] = win[k];
}

// Convolution + SiLU of every (token, channel) of a mamba block, in parallel: value[t][c] from the entry
// rows t - taps + 1 .. t (the block's conv window before the chunk for the first tokens).
__global__ void __launch_bounds__(kThreads) ssm_value_kernel(IvbLayerDesc L, const float* ent, int T, int d, int ld, int taps,
                                                             float* value) {
  const int i = blockIdx.x * kThreads + threadIdx.x;
  if (i >= T * d) return;
  const int t = i / d, c = i - t * d;
  float conv = L.conv_bias[c];
  for (int k2 = 0; k2 < taps; ++k2) {
    const int src = t - (taps - 1) + k2;  // token index of tap k2 (negative: the stored window)
    const float x = src >= 0 ? ent[static_cast<size_t>(src) * ld + c] : L.conv_state[static_cast<size_t>(c) * (taps - 1) + (taps - 1 + src)];
    conv = fmaf(L.conv_weight[c * taps + k2], x, conv);
  }
  value[i] = silu_f(conv);
}

// Recurrent scan over the tokens with the per-(token, head, state) coefficients computed cooperatively
// for blocks of 32 tokens into shared memory. CTA: 16 channels x 16 state lanes (lane s of a channel's
// half-warp owns state s). The conv window of the block is advanced at the end. Same arithmetic per
// step as the decode kernel.
constexpr int kScanBlock = 32;
__global__ void __launch_bounds__(kThreads) ssm_scan_block_kernel(IvbLayerDesc L, const float* ent, const float* value, int T,
                                                                  int d, int H, int hd, int S, int taps, float half_dt_min,
                                                                  float half_dt_range, float* y) {
  extern __shared__ float sh[];
  const int tid = threadIdx.x, sub = tid & 15, chl = tid >> 4;
  const int c0 = blockIdx.x * 16, c = c0 + chl;
  const bool live = c < d;
  const int h0 = c0 / hd, nhc = (min(d, c0 + 16) - 1) / hd - h0 + 1;  // heads spanned by the CTA's channels
  float* coef = sh;                                   // [kScanBlock][nhc][S][5]
  float* vals = coef + kScanBlock * nhc * S * 5;      // [kScanBlock][16]
  float* gates = vals + kScanBlock * 16;              // [kScanBlock][16]
  const int ld = 2 * d + 3 * H * S;
  const int h = live ? c / hd : h0, dd = live ? c - h * hd : 0;
  const bool on = live && sub < S;
  const int s = on ? sub : 0;
  const size_t si_idx = (static_cast<size_t>(h) * S + s) * hd + dd;
  float sr = on ? L.ssm_state[2 * si_idx] : 0.0f, si = on ? L.ssm_state[2 * si_idx + 1] : 0.0f;
  float prev = on ? L.prev_force[si_idx] : 0.0f;
  const float skip = live ? L.skip[c] : 0.0f;
  for (int t0 = 0; t0 < T; t0 += kScanBlock) {
    const int nt = min(kScanBlock, T - t0);
    __syncthreads();
    for (int idx = tid; idx < nt * nhc * S; idx += kThreads) {
      const int tt = idx / (nhc * S), rest = idx - tt * (nhc * S), hl = rest / S, s2 = rest - hl * S;
      const int hh = h0 + hl;
      const float* bcdt = ent + static_cast<size_t>(t0 + tt) * ld + 2 * d + hh * 3 * S;
      const float half_dt = half_dt_min + sigmoid_f(bcdt[2 * S + s2]) * half_dt_range;
      const float mag = expf(2.0f * half_dt * L.decay[hh * S + s2]);
      float sn, cs;
      sincosf(2.0f * half_dt * L.theta[hh * S + s2], &sn, &cs);
      float* cf = coef + (static_cast<size_t>(tt) * nhc * S + hl * S + s2) * 5;
      cf[0] = tanhf(bcdt[s2]);
      cf[1] = tanhf(bcdt[S + s2]);
      cf[2] = half_dt;
      cf[3] = mag * cs;
      cf[4] = mag * sn;
    }
    for (int idx = tid; idx < nt * 16; idx += kThreads) {
      const int tt = idx >> 4, ch = idx & 15;
      const int cc2 = c0 + ch;
      vals[idx] = cc2 < d ? value[static_cast<size_t>(t0 + tt) * d + cc2] : 0.0f;
      gates[idx] = cc2 < d ? ent[static_cast<size_t>(t0 + tt) * ld + d + cc2] : 0.0f;
    }
    __syncthreads();
    const int hl = h - h0;
    for (int tt = 0; tt < nt; ++tt) {
      const float v = vals[tt * 16 + chl];
      float contrib = 0.0f;
      if (on) {
        const float* cf = coef + (static_cast<size_t>(tt) * nhc * S + hl * S + s) * 5;
        const float b = cf[0], cc = cf[1], half_dt = cf[2], ar = cf[3], ai = cf[4];
        const float force = b * v;
        const float dr = (force + ar * prev) * half_dt;
        const float di = (ai * prev) * half_dt;
        const float nr = sr * ar - si * ai + dr;
        const float ni = sr * ai + si * ar + di;
        sr = nr;
        si = ni;
        prev = force;
        contrib = cc * nr;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) contrib += __shfl_xor_sync(kFull, contrib, off);
      if (live && sub == 0)
        y[static_cast<size_t>(t0 + tt) * d + c] = (contrib + skip * v) * sigmoid_f(gates[tt * 16 + chl]);
    }
  }
  if (on) {
    L.ssm_state[2 * si_idx] = sr;
    L.ssm_state[2 * si_idx + 1] = si;
    L.prev_force[si_idx] = prev;
  }
  // the conv window after the last token: the last taps - 1 inputs (older window entries when T is short)
  __syncthreads();
  if (live && sub == 0) {
    float w[kMaxTaps];
    for (int k = 0; k < taps - 1; ++k) {
      const int src = T - (taps - 1) + k;
      w[k] = src >= 0 ? ent[static_cast<size_t>(src) * ld + c] : L.conv_state[static_cast<size_t>(c) * (taps - 1) + (taps - 1 + src)];
    }
    for (int k = 0; k < taps - 1; ++k) L.conv_state[static_cast<size_t>(c) * (taps - 1) + k] = w[k];
  }
}

// Cache fill of one mla block for T tokens at positions pos0..: the quantised latent and the rotated,
// fp16-rounded k_rope of every head. One CTA per token. ent [T][d + Lt + H*rope]: q | latent | k_rope.
__global__ void __launch_bounds__(kThreads) mla_cache_kernel(IvbLayerDesc L, const float* ent, int pos0, int d, int Lt,
                                                             int H, int rope, int max_len, int lpad, int rpad, float act_eps) {
  __shared__ float xl[512 + 64];
  __shared__ __align__(16) int8_t codes[576];
  __shared__ float red[64];
  const int t = blockIdx.x, pos = pos0 + t;
  const int ld = d + Lt + H * rope;
  const float* row = ent + static_cast<size_t>(t) * ld;
  for (int j = threadIdx.x; j < Lt; j += kThreads) xl[j] = row[d + j];
  __syncthreads();
  const float a = quantize_block(xl, Lt, nullptr, 0.0f, 0.0f, act_eps, codes, false, nullptr, red);
  for (int j = threadIdx.x; j < Lt; j += kThreads) L.latent_q[static_cast<size_t>(pos) * lpad + j] = codes[j];
  if (threadIdx.x == 0) L.latent_scale[pos] = a;
  const float* rtab = L.rope + static_cast<size_t>(pos) * rope;
  for (int i = threadIdx.x; i < H * (rope / 2); i += kThreads) {
    const int h = i / (rope / 2), jr = i - h * (rope / 2);
    const float cs = __ldg(rtab + 2 * jr), sn = __ldg(rtab + 2 * jr + 1);
    const float k0 = row[d + Lt + h * rope + 2 * jr], k1 = row[d + Lt + h * rope + 2 * jr + 1];
    uint16_t* kc = L.k_rope_cache + (static_cast<size_t>(h) * max_len + pos) * rpad;
    kc[2 * jr] = f2h(k0 * cs - k1 * sn);
    kc[2 * jr + 1] = f2h(k0 * sn + k1 * cs);
  }
}

// Causal latent attention of token t (position pos0 + t) and head h over cached positions 0..pos0+t.
// Absorbed form as in the decode kernel: s_p = a_p <qa, ql_p> + q_nope.b_k + <q_rope, k_rope_p>, online
// softmax, u = sum p_p a_p ql_p, out = W_v u / l + b_v. 128 threads; 8 lanes per position for scores,
// a warp per position group for u.
constexpr int kAttnThreads = 128;
constexpr int kAttnTile = 128;

__global__ void __launch_bounds__(kAttnThreads) mla_attention_kernel(IvbLayerDesc L, const float* ent, int pos0, int d, int Lt,
                                                                     int H, int hd, int rope, int nope, int max_len, int lpad,
                                                                     int rpad, float* y) {
  __shared__ float qa[512];
  __shared__ float qn[256];
  __shared__ float qr[128];
  __shared__ float sc[kAttnTile];
  __shared__ float part[4][512];
  __shared__ float red[64];
  const int t = blockIdx.x, h = blockIdx.y, pos = pos0 + t;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ld = d + Lt + H * rope;
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
  // absorbed query
  const IvbTernary& kn = L.k_nope_up;
  for (int j = tid; j < Lt; j += kAttnThreads) {
    float acc = 0.0f;
    for (int e = 0; e < nope; ++e) {
      const size_t r = static_cast<size_t>(h) * nope + e;
      acc = fmaf(qn[e], code_value(kn.packed + r * kn.row_bytes, j) * h2f(__ldg(kn.scales + r * kn.scale_stride + (j >> 7))), acc);
    }
    qa[j] = acc;
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
      const int8_t* ql = L.latent_q + static_cast<size_t>(p) * lpad;
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
      const uint16_t* kr = L.k_rope_cache + (static_cast<size_t>(h) * max_len + p) * rpad;
      for (int r = sub; r < rope; r += 8) rp = fmaf(qr[r], h2f(__ldcg(kr + r)), rp);
      float total = fmaf(__ldcg(L.latent_scale + p), dot, rp);
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
      sc[k] = e * __ldcg(L.latent_scale + start + k);
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
      const int8_t* ql = L.latent_q + static_cast<size_t>(start + k) * lpad;
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
  const IvbTernary& vu = L.v_up;
  const float inv_l = 1.0f / l_run;
  for (int e = tid; e < hd; e += kAttnThreads) {
    const size_t r = static_cast<size_t>(h) * hd + e;
    float acc = 0.0f;
    for (int j = 0; j < Lt; ++j)
      acc = fmaf(code_value(vu.packed + r * vu.row_bytes, j) * h2f(__ldg(vu.scales + r * vu.scale_stride + (j >> 7))), qa[j], acc);
    float o = acc * inv_l;
    if (vu.bias != nullptr) o += __ldg(vu.bias + r);
    y[static_cast<size_t>(t) * d + h * hd + e] = o;
  }
}

__global__ void prefill_finish_kernel(const int64_t* tokens, int count, int pos_end, int64_t* token, int64_t* position) {
  token[0] = tokens[count - 1];
  position[0] = pos_end;
}

struct PrefillLayout {
  size_t resid, ent, y, h, q8, scale, err, total;
  int ldq, groups, ld_ent;
};

static PrefillLayout prefill_layout(const IvbModelDesc& md, const IvbLayerDesc* layers, int max_tokens) {
  PrefillLayout L{};
  const int d = md.hidden, F = md.dense;
  int ld_ent = 0;
  for (int i = 0; i < md.num_layers; ++i) ld_ent = std::max(ld_ent, layers[i].entry.rows);
  L.ld_ent = ld_ent;
  L.ldq = (std::max(d, F) + 127) / 128 * 128;
  L.groups = L.ldq / 128;
  const size_t T = static_cast<size_t>(max_tokens);
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  L.resid = take(T * d * 4);
  L.ent = take(T * ld_ent * 4);
  L.y = take(T * d * 4);
  L.h = take(T * std::max(F, d) * 4);  // also the mamba conv values [T][d]
  L.q8 = take((T + 127) / 128 * 128 * L.ldq);  // whole 128-token tiles
  L.scale = take(T * 4);
  L.err = take(16);
  L.total = o;
  return L;
}

}  // namespace ivb

extern "C" {

uint64_t ivb_decoder_prefill_workspace_bytes(const IvbDecoder* dec, int32_t max_tokens) {
  using namespace ivb;
  if (dec == nullptr || max_tokens <= 0) return 0;
  const IvbLayerDesc* layers = nullptr;
  const IvbModelDesc& md = decoder_model(dec, &layers);
  return prefill_layout(md, layers, max_tokens).total;
}

int32_t ivb_decoder_prefill(IvbDecoder* dec, const int64_t* tokens, int32_t count, int32_t start_position, void* workspace,
                            uint64_t workspace_bytes, void* stream) {
  using namespace ivb;
  if (dec == nullptr || tokens == nullptr || workspace == nullptr) return fail(IVB_EINVAL, "ivb_decoder_prefill: null argument");
  const IvbLayerDesc* layers = nullptr;
  const IvbModelDesc& md = decoder_model(dec, &layers);
  if (count <= 0) return fail(IVB_EINVAL, "ivb_decoder_prefill: count must be positive");
  if (start_position < 0 || start_position + count > md.max_len)
    return fail(IVB_ECAPACITY, "ivb_decoder_prefill: %d tokens at position %d exceed the capacity %d", count, start_position,
                md.max_len);
  const PrefillLayout W = prefill_layout(md, layers, count);
  if (workspace_bytes < W.total) return fail(IVB_EINVAL, "ivb_decoder_prefill: workspace too small (%llu < %zu)",
                                             static_cast<unsigned long long>(workspace_bytes), W.total);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return fail(IVB_EINVAL, "ivb_decoder_prefill: workspace must be 256-byte aligned");
  const int d = md.hidden, F = md.dense, H = md.heads, hd = md.head_dim, S = md.state_dim, Lt = md.latent_dim;
  const int rope = md.rope_dim, nope = md.nope_dim;
  if (Lt > 512 || rope > 128 || nope > 256) return fail(IVB_EINVAL, "ivb_decoder_prefill: latent/rope/nope beyond the prefill kernels");
  for (int i = 0; i < md.num_layers; ++i)
    if (layers[i].kind == IVB_MAMBA && (layers[i].conv_taps > kMaxTaps + 1 || S > 16))
      return fail(IVB_EINVAL, "ivb_decoder_prefill: conv width %d or state %d beyond the scan kernel", layers[i].conv_taps, S);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  float* resid = reinterpret_cast<float*>(ws + W.resid);
  float* ent = reinterpret_cast<float*>(ws + W.ent);
  float* y = reinterpret_cast<float*>(ws + W.y);
  float* hbuf = reinterpret_cast<float*>(ws + W.h);
  int8_t* q8 = reinterpret_cast<int8_t*>(ws + W.q8);
  float* scale = reinterpret_cast<float*>(ws + W.scale);
  uint32_t* err = decoder_error_word(dec);  // reported by ivb_decoder_check
  if (err == nullptr) return fail(IVB_EINVAL, "ivb_decoder_prefill: bind the decoder first");
  const int lpad = static_cast<int>((Lt + 15) / 16 * 16), rpad = (rope + 7) / 8 * 8;
  embed_rows_kernel<<<count, kThreads, 0, s>>>(md.head, tokens, d, resid);
  IVB_CUDA(cudaGetLastError());
  auto quant = [&](const float* x, int n, const float* norm, float eps) -> int32_t {
    const int ld = (n + 127) / 128 * 128;
    return ivb_quantize_rows(x, count, n, norm, eps, md.norm_clip, md.act_eps, q8, ld, scale, nullptr, stream);
  };
  auto gemm = [&](const IvbTernary& m, int epilogue, float* out, int ldo) -> int32_t {
    const int ld = (m.in_features + 127) / 128 * 128;
    return ivb_ternary_gemm(&m, q8, ld, scale, count, epilogue, out, ldo, err, stream);
  };
  for (int li = 0; li < md.num_layers; ++li) {
    const IvbLayerDesc& L = layers[li];
    if (int32_t rc = quant(resid, d, L.mixer_norm, L.mixer_norm_eps)) return rc;
    if (int32_t rc = gemm(L.entry, IVB_EPI_STORE, ent, L.entry.rows)) return rc;
    if (L.kind == IVB_MAMBA && hd >= 4) {
      const int ld = 2 * d + 3 * H * S;
      ssm_value_kernel<<<(count * d + kThreads - 1) / kThreads, kThreads, 0, s>>>(L, ent, count, d, ld, L.conv_taps, hbuf);
      IVB_CUDA(cudaGetLastError());
      const int nhc_max = std::min(16, 15 / hd + 2);
      const size_t smem = (static_cast<size_t>(kScanBlock) * nhc_max * S * 5 + 2 * kScanBlock * 16) * 4;
      IVB_CUDA(cudaFuncSetAttribute(ssm_scan_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
      ssm_scan_block_kernel<<<(d + 15) / 16, kThreads, smem, s>>>(L, ent, hbuf, count, d, H, hd, S, L.conv_taps, L.half_dt_min,
                                                                   L.half_dt_range, y);
      IVB_CUDA(cudaGetLastError());
    } else if (L.kind == IVB_MAMBA) {
      const int blocks = (d * 16 + kThreads - 1) / kThreads;
      ssm_scan_kernel<<<blocks, kThreads, 0, s>>>(L, ent, count, d, H, hd, S, L.conv_taps, L.half_dt_min, L.half_dt_range, y);
      IVB_CUDA(cudaGetLastError());
    } else {
      mla_cache_kernel<<<count, kThreads, 0, s>>>(L, ent, start_position, d, Lt, H, rope, md.max_len, lpad, rpad, md.act_eps);
      IVB_CUDA(cudaGetLastError());
      mla_attention_kernel<<<dim3(count, H), kAttnThreads, 0, s>>>(L, ent, start_position, d, Lt, H, hd, rope, nope,
                                                                  md.max_len, lpad, rpad, y);
      IVB_CUDA(cudaGetLastError());
    }
    if (int32_t rc = quant(y, d, nullptr, 0.0f)) return rc;
    if (int32_t rc = gemm(L.out, IVB_EPI_RESIDUAL, resid, d)) return rc;
    if (int32_t rc = quant(resid, d, L.ffn_norm, L.ffn_norm_eps)) return rc;
    if (int32_t rc = gemm(L.gate_up, IVB_EPI_SILU_PAIR, hbuf, F)) return rc;
    if (int32_t rc = quant(hbuf, F, nullptr, 0.0f)) return rc;
    if (int32_t rc = gemm(L.down, IVB_EPI_RESIDUAL, resid, d)) return rc;
  }
  // the head on the last token
  if (int32_t rc = ivb_ternary_gemv(&md.head, resid + static_cast<size_t>(count - 1) * d, md.final_norm, md.final_norm_eps,
                                    md.norm_clip, md.act_eps, IVB_EPI_STORE, md.logits, stream))
    return rc;
  prefill_finish_kernel<<<1, 1, 0, s>>>(tokens, count, start_position + count, md.token, md.position);
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

}  // extern "C"
