// Prompt prefill of libivonar_b200.so: all prompt tokens of a chunk go through each layer together.
//
// Per block: quantise every token row (ivb_quantize_rows), the entry projection as one tcgen05 int8
// GEMM over all tokens (ivb_ternary_gemm), then the mixer, then the out, gate/up and down GEMMs with
// their residual / SwiGLU epilogues. Mamba mixer: the convolution values of all tokens in parallel,
// then the recurrence over the tokens with the per-token coefficients staged in shared memory for
// blocks of 32 tokens. MLA mixer: the latent/k_rope cache fill of every token, the per-head keys and
// values of all cached positions from the latent (two more tcgen05 GEMMs), then causal flash attention
// on tensor cores. The head runs on the last token only. Caches, recurrent state, position and token
// end exactly where the token-by-token decode kernel would leave them, so decoding continues from
// here. Replaces kernel_decoder.py:457-479 (prefill) and kernels/ternary.cu:688-982 (tile GEMM,
// recurrent tile, kv write, attention tile).
#include <cuda_runtime.h>

#include <algorithm>

#include "ivb_common.h"
#include "ivb_decode.cuh"
#include "ivb_tiles.cuh"

namespace ivb {


constexpr int kMaxTaps = 8;

// Embedding rows of the prompt tokens (the tied head): resid[t][i] = (code - 1) * scale.
__global__ void __launch_bounds__(kThreads) embed_rows_kernel(IvbTernary head, const int64_t* tokens, int d, float* resid) {
  pdl_enter();
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
  pdl_enter();
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
  pdl_enter();
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

// Per-(token, head, state) coefficients of the recurrence, all tokens in parallel:
// coef[t][h][s] = (tanh B, tanh C, half_dt, Re alpha, Im alpha) with alpha = exp(2 half_dt (decay + i theta)).
__global__ void ssm_coef_kernel(IvbLayerDesc L, const float* ent, int T, int d, int H, int S, int ld, float half_dt_min,
                                float half_dt_range, float* coefb) {
  pdl_enter();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * H * S) return;
  const int t = i / (H * S), rest = i - t * (H * S), h = rest / S, s = rest - h * S;
  const float* bcdt = ent + static_cast<size_t>(t) * ld + 2 * d + h * 3 * S;
  const float half_dt = half_dt_min + sigmoid_f(bcdt[2 * S + s]) * half_dt_range;
  const float mag = expf(2.0f * half_dt * L.decay[h * S + s]);
  float sn, cs;
  sincosf(2.0f * half_dt * L.theta[h * S + s], &sn, &cs);
  float* cf = coefb + static_cast<size_t>(i) * 5;
  cf[0] = tanhf(bcdt[s]);
  cf[1] = tanhf(bcdt[S + s]);
  cf[2] = half_dt;
  cf[3] = mag * cs;
  cf[4] = mag * sn;
}

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

// Chunked scan. The recurrence is linear in the state: x_t = a_t x_{t-1} + u_t with
// u_t = half_dt_t (f_t + a_t f_{t-1}) (f = B v, the force, an input), so the tokens split into chunks
// of kScanChunk that run in parallel: each chunk scans from a zero state (its x~_t), the chunk-local
// products A_t = a_first..a_t (ssm_cumprod_kernel) carry a chunk's start state to every token, a short
// pass over the chunks (ssm_carry_kernel) finds each chunk's start state, and ssm_output_kernel adds
// C_t Re(A_t x_start) to the chunk's partial output and applies skip and gate:
//   x_t = x~_t + A_t x_start(chunk of t).
// The per-step arithmetic is the decode step's; only the grouping of the state sums differs.
//
// Chunk scan (grid: channel groups x chunks): blocks of 32 tokens, the block's coefficients
// (ssm_coef_kernel), conv values (ssm_value_kernel) copied into shared memory with cp.async one block
// ahead, the recurrence with one lane per state, the 16-lane sums afterwards for the whole block
// (written to y as the partial output). CTA: 16 channels x 16 state lanes.
constexpr int kScanBlock = 32;
constexpr int kScanChunk = 128;            // tokens per chunk (a multiple of kScanBlock)
constexpr int kScanCh = 16;                // channels per CTA
constexpr int kScanThreads = 16 * kScanCh;
__global__ void __launch_bounds__(kScanThreads) ssm_scan_block_kernel(IvbLayerDesc L, const float* ent, const float* value,
                                                                  const float* coefb, int T, int d, int H, int hd, int S,
                                                                  int taps, float* xend, float* y) {
  pdl_enter();
  extern __shared__ float sh[];
  const int tid = threadIdx.x, sub = tid & 15, chl = tid >> 4;
  const int c0 = blockIdx.x * kScanCh, c = c0 + chl;
  const bool live = c < d;
  const int h0 = c0 / hd, nhc = (min(d, c0 + kScanCh) - 1) / hd - h0 + 1;  // heads spanned by the CTA's channels
  const int per_blk = kScanBlock * nhc * S * 5 + kScanBlock * kScanCh;  // coef | vals
  float* ctb = sh + 2 * per_blk;                                            // [kScanBlock][threads]: C * Re(state)
  const int ld = 2 * d + 3 * H * S;
  const int h = live ? c / hd : h0, dd = live ? c - h * hd : 0;
  const bool on = live && sub < S;
  const int s = on ? sub : 0;
  const size_t si_idx = (static_cast<size_t>(h) * S + s) * hd + dd;
  const int t_begin = blockIdx.y * kScanChunk, t_end = min(T, t_begin + kScanChunk);
  const bool last_chunk = t_end == T;
  // every chunk scans from a zero state; the force before the chunk is an input (or the stored one)
  float sr = 0.0f, si = 0.0f, prev = 0.0f;
  if (on) {
    if (t_begin == 0) {
      prev = L.prev_force[si_idx];
    } else {
      const float* cfp = coefb + ((static_cast<size_t>(t_begin - 1) * H + h) * S + s) * 5;
      prev = cfp[0] * value[static_cast<size_t>(t_begin - 1) * d + c];
    }
  }
  auto prefetch = [&](int t0, float* buf) {
    const int nt = min(kScanBlock, T - t0);
    float* coef = buf;
    float* vals = coef + kScanBlock * nhc * S * 5;
    const int row = nhc * S * 5;  // coefficients of the CTA's heads for one token, contiguous
    for (int idx = tid; idx < nt * row; idx += kScanThreads) {
      const int tt = idx / row, k = idx - tt * row;
      cp_async4(coef + idx, coefb + (static_cast<size_t>(t0 + tt) * H + h0) * S * 5 + k);
    }
    for (int idx = tid; idx < nt * kScanCh; idx += kScanThreads) {
      const int tt = idx / kScanCh, cc2 = c0 + (idx % kScanCh);
      if (cc2 < d) cp_async4(vals + idx, value + static_cast<size_t>(t0 + tt) * d + cc2);
      else vals[idx] = 0.0f;
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  prefetch(t_begin, sh);
  for (int t0 = t_begin, blk = 0; t0 < t_end; t0 += kScanBlock, ++blk) {
    const int nt = min(kScanBlock, t_end - t0);
    float* buf = sh + (blk & 1) * per_blk;
    const float* coef = buf;
    const float* vals = coef + kScanBlock * nhc * S * 5;
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // this block's data has landed; the other buffer and ctb are free
    if (t0 + kScanBlock < t_end) prefetch(t0 + kScanBlock, sh + ((blk + 1) & 1) * per_blk);
    const int hl = h - h0;
    const float* cf0 = coef + (hl * S + s) * 5;
    const int cstep = nhc * S * 5;
    // the recurrence alone stays on the sequential path; the per-channel sums over the state lanes and
    // the output gate run afterwards for the whole block
#pragma unroll 4
    for (int tt = 0; tt < nt; ++tt) {
      const float v = vals[tt * kScanCh + chl];
      float contrib = 0.0f;
      if (on) {
        const float* cf = cf0 + tt * cstep;
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
      ctb[tt * kScanThreads + tid] = contrib;
    }
    __syncthreads();
    for (int idx = tid; idx < nt * kScanCh; idx += kScanThreads) {
      const int tt = idx / kScanCh, ch = idx % kScanCh, cc2 = c0 + ch;
      if (cc2 >= d) continue;
      // the xor-butterfly order of the decode kernel's 16-lane warp sum (offsets 8, 4, 2, 1), lane 0
      const float* v = ctb + tt * kScanThreads + ch * 16;
      float a[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = v[i] + v[i + 8];
      const float sum = ((a[0] + a[4]) + (a[2] + a[6])) + ((a[1] + a[5]) + (a[3] + a[7]));
      y[static_cast<size_t>(t0 + tt) * d + cc2] = sum;  // partial output, finished by ssm_output_kernel
    }
  }
  if (on) {
    const size_t xo = (static_cast<size_t>(blockIdx.y) * H * S * hd + si_idx) * 2;
    xend[xo] = sr;
    xend[xo + 1] = si;
    if (last_chunk) L.prev_force[si_idx] = prev;
  }
  // the conv window after the last token: the last taps - 1 inputs (older window entries when T is short)
  __syncthreads();
  if (last_chunk && live && sub == 0) {
    float w[kMaxTaps];
    for (int k = 0; k < taps - 1; ++k) {
      const int src = T - (taps - 1) + k;
      w[k] = src >= 0 ? ent[static_cast<size_t>(src) * ld + c] : L.conv_state[static_cast<size_t>(c) * (taps - 1) + (taps - 1 + src)];
    }
    for (int k = 0; k < taps - 1; ++k) L.conv_state[static_cast<size_t>(c) * (taps - 1) + k] = w[k];
  }
}

// Chunk-local products of the decay factors: A[t][h][s] = a_first(chunk) ... a_t (complex), one thread
// per (chunk, head, state).
__global__ void ssm_cumprod_kernel(const float* coefb, int T, int H, int S, float* cum) {
  pdl_enter();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int chunks = (T + kScanChunk - 1) / kScanChunk;
  if (i >= chunks * H * S) return;
  const int k = i / (H * S), hs = i - k * (H * S);
  float pr = 1.0f, pi = 0.0f;
  const int t_end = min(T, (k + 1) * kScanChunk);
  // the coefficients of 16 tokens are loaded before their products are stored, so the loads overlap
  // (stores into cum could alias coefb as far as the compiler knows)
  constexpr int kBatch = 16;
  for (int t0 = k * kScanChunk; t0 < t_end; t0 += kBatch) {
    float ar[kBatch], ai[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int t = t0 + j;
      ar[j] = ai[j] = 0.0f;
      if (t < t_end) {
        const float* cf = coefb + (static_cast<size_t>(t) * H * S + hs) * 5;
        ar[j] = cf[3];
        ai[j] = cf[4];
      }
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int t = t0 + j;
      if (t < t_end) {
        const float nr = pr * ar[j] - pi * ai[j], ni = pr * ai[j] + pi * ar[j];
        pr = nr;
        pi = ni;
        cum[(static_cast<size_t>(t) * H * S + hs) * 2] = pr;
        cum[(static_cast<size_t>(t) * H * S + hs) * 2 + 1] = pi;
      }
    }
  }
}

// Start state of every chunk, one thread per (head, state, channel): x_start(0) = the stored state,
// x_start(k + 1) = x~_end(k) + A_end(k) x_start(k); the state after the last token is stored.
__global__ void ssm_carry_kernel(IvbLayerDesc L, const float* cum, const float* xend, int T, int H, int S, int hd,
                                 float* carry) {
  pdl_enter();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int lanes = H * S * hd;
  if (i >= lanes) return;
  const int hs = i / hd;  // (h * S + s)
  const int chunks = (T + kScanChunk - 1) / kScanChunk;
  float xr = L.ssm_state[2 * static_cast<size_t>(i)], xi = L.ssm_state[2 * static_cast<size_t>(i) + 1];
  // the inputs of 8 chunks are loaded before their carries are stored, so the loads overlap
  constexpr int kBatch = 8;
  for (int k0 = 0; k0 < chunks; k0 += kBatch) {
    float ar[kBatch], ai[kBatch], er[kBatch], ei[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int k = k0 + j;
      ar[j] = ai[j] = er[j] = ei[j] = 0.0f;
      if (k < chunks) {
        const int t_last = min(T, (k + 1) * kScanChunk) - 1;
        ar[j] = cum[(static_cast<size_t>(t_last) * H * S + hs) * 2];
        ai[j] = cum[(static_cast<size_t>(t_last) * H * S + hs) * 2 + 1];
        er[j] = xend[(static_cast<size_t>(k) * lanes + i) * 2];
        ei[j] = xend[(static_cast<size_t>(k) * lanes + i) * 2 + 1];
      }
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int k = k0 + j;
      if (k < chunks) {
        carry[(static_cast<size_t>(k) * lanes + i) * 2] = xr;
        carry[(static_cast<size_t>(k) * lanes + i) * 2 + 1] = xi;
        const float nr = er[j] + (ar[j] * xr - ai[j] * xi), ni = ei[j] + (ar[j] * xi + ai[j] * xr);
        xr = nr;
        xi = ni;
      }
    }
  }
  L.ssm_state[2 * static_cast<size_t>(i)] = xr;
  L.ssm_state[2 * static_cast<size_t>(i) + 1] = xi;
}

// y[t][c] = (partial + sum_s C_t Re(A_t x_start) + skip v_t) * sigmoid(gate_t), one thread per (t, c);
// the sum over the states in the decode kernel's xor-butterfly order.
__global__ void ssm_output_kernel(IvbLayerDesc L, const float* ent, const float* value, const float* coefb, const float* cum,
                                  const float* carry, int T, int d, int H, int hd, int S, float* y) {
  pdl_enter();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * d) return;
  const int t = i / d, c = i - t * d, h = c / hd, dd = c - h * hd;
  const int k = t / kScanChunk;
  const int lanes = H * S * hd;
  const int ld = 2 * d + 3 * H * S;
  float v[16];
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    v[s] = 0.0f;
    if (s < S) {
      const size_t hs = static_cast<size_t>(h) * S + s;
      const float cc = coefb[(static_cast<size_t>(t) * H * S + hs) * 5 + 1];
      const float ar = cum[(static_cast<size_t>(t) * H * S + hs) * 2], ai = cum[(static_cast<size_t>(t) * H * S + hs) * 2 + 1];
      const size_t ci = (static_cast<size_t>(k) * lanes + hs * hd + dd) * 2;
      v[s] = cc * (ar * carry[ci] - ai * carry[ci + 1]);
    }
  }
  float a[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] = v[j] + v[j + 8];
  const float corr = ((a[0] + a[4]) + (a[2] + a[6])) + ((a[1] + a[5]) + (a[3] + a[7]));
  const float* row = ent + static_cast<size_t>(t) * ld;
  y[i] = ((y[i] + corr) + __ldg(L.skip + c) * value[i]) * sigmoid_f(row[d + c]);
}

// Cache fill of one mla block for T tokens at positions pos0..: the quantised latent and the rotated,
// fp16-rounded k_rope of every head. One CTA per token. ent [T][d + Lt + H*rope]: q | latent | k_rope.
__global__ void __launch_bounds__(kThreads) mla_cache_kernel(IvbLayerDesc L, const float* ent, int pos0, int d, int Lt,
                                                             int H, int rope, int max_len, int lpad, int rpad, float act_eps) {
  pdl_enter();
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

// ---- causal attention of the prefill on tensor cores ---------------------------------------------
// Non-absorbed form: the cached latent of every position p (int8 codes ql_p, scale a_p) is expanded
// by the tcgen05 GEMM into per-head keys K_nope[p] = a_p W_k ql_p + b_k and values V[p] = a_p W_v ql_p
// + b_v, which is the same arithmetic as the decode kernel's absorbed form regrouped:
// a_p <W_k^T q, ql_p> + q.b_k = q.K_nope[p] and W_v (sum_p w_p a_p ql_p) + b_v = sum_p w_p V[p] (the
// weights w sum to one). Then a flash-attention kernel per (64-token query block, head) runs
// mma.sync m16n8k16 with fp16 operands in a three-product split (x = hi + lo, x.y ~ hi.hi' + hi.lo' +
// lo.hi'), which keeps about 22 significant bits, close to the fp32 arithmetic of the decode path.

// Latent codes of positions 0..P-1 into the tiled GEMM activation layout (ldq = latent rounded to 128).
__global__ void latent_tile_kernel(const int8_t* latent_q, int lpad, int Lt, int P, int ldq, int8_t* q8) {
  pdl_enter();
  const int chunks = ldq >> 4;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P * chunks) return;
  const int p = i / chunks, k = i - p * chunks;
  // byte 4f + b of the chunk holds input 16k + 4b + f
  uint32_t o[4];
#pragma unroll
  for (int f = 0; f < 4; ++f) {
    uint32_t w = 0u;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int j = (k << 4) + 4 * b + f;
      w |= (j < Lt ? static_cast<uint32_t>(static_cast<uint8_t>(latent_q[static_cast<size_t>(p) * lpad + j])) : 0u) << (8 * b);
    }
    o[f] = w;
  }
  *reinterpret_cast<uint4*>(q8 + q8_chunk_offset(p, k, ldq)) = make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// x = hi + lo with hi, lo fp16 (packed pairs)
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
  const __half l0 = __float2half_rn(x0 - __half2float(h0)), l1 = __float2half_rn(x1 - __half2float(h1));
  hi = static_cast<uint32_t>(__half_as_ushort(h0)) | (static_cast<uint32_t>(__half_as_ushort(h1)) << 16);
  lo = static_cast<uint32_t>(__half_as_ushort(l0)) | (static_cast<uint32_t>(__half_as_ushort(l1)) << 16);
}

constexpr int kFaTok = 64;      // query tokens per CTA (4 warps x 16)
constexpr int kFaPos = 64;      // key positions per tile
constexpr int kFaThreads = 128;

// Keys and values of positions 0..P-1 of one layer as fp16 hi/lo pairs, laid out for whole-tile copies:
// kh/kl [H][Ppad][DK] (K_nope then k_rope, zero padded), vh/vl [H][DV][Ppad] (transposed, zero padded),
// Ppad = P rounded up to kFaPos. One thread per (head, position, 8 dims).
template <int DK>
__global__ void kv_split_kernel(IvbLayerDesc L, const float* knope, const float* vbuf, int P, int Ppad, int d, int H,
                                int hd, int rope, int nope, int max_len, int rpad, __half* kh, __half* kl, __half* vh,
                                __half* vl) {
  pdl_enter();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int per_head = Ppad * (DK / 8);
  if (i >= H * per_head) return;
  const int h = i / per_head, rest = i - h * per_head, p = rest / (DK / 8), e0 = (rest - p * (DK / 8)) * 8;
  uint32_t khw[4], klw[4], vhw[8], vlw[8];
  float kv[8], vv[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int e = e0 + j;
    float k = 0.0f, v = 0.0f;
    if (p < P) {
      if (e < nope) k = knope[static_cast<size_t>(p) * H * nope + h * nope + e];
      else if (e < nope + rope) k = h2f(L.k_rope_cache[(static_cast<size_t>(h) * max_len + p) * rpad + (e - nope)]);
      if (e < hd) v = vbuf[static_cast<size_t>(p) * d + h * hd + e];
    }
    kv[j] = k;
    vv[j] = v;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) split2(kv[2 * j], kv[2 * j + 1], khw[j], klw[j]);
  const size_t ko = (static_cast<size_t>(h) * Ppad + p) * DK + e0;
  *reinterpret_cast<uint4*>(kh + ko) = make_uint4(khw[0], khw[1], khw[2], khw[3]);
  *reinterpret_cast<uint4*>(kl + ko) = make_uint4(klw[0], klw[1], klw[2], klw[3]);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (e0 + j >= DK) break;
    const __half hv = __float2half_rn(vv[j]);
    const size_t vo = (static_cast<size_t>(h) * DK + e0 + j) * Ppad + p;
    vh[vo] = hv;
    vl[vo] = __float2half_rn(vv[j] - __half2float(hv));
  }
  (void)vhw;
  (void)vlw;
}

// The decode kernel's key / value cache rows of positions pos0 .. pos0 + T - 1 (layout of
// IvbLayerDesc.k_cache / v_cache): keys [K_nope | rotated k_rope as k_rope_cache holds it], values, zero
// padding to kvpad floats. One thread per (position, head, dim).
__global__ void kv_cache_kernel(IvbLayerDesc L, const float* knope, const float* vbuf, int pos0, int T, int H, int hd, int nope,
                                int max_len, int rpad, int kvpad) {
  pdl_enter();
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(T) * H * kvpad) return;
  const int e = static_cast<int>(i % kvpad);
  const long long r = i / kvpad;
  const int h = static_cast<int>(r % H), pos = pos0 + static_cast<int>(r / H);
  float k = 0.0f, v = 0.0f;
  if (e < nope) k = knope[static_cast<size_t>(pos) * H * nope + h * nope + e];
  else if (e < hd) k = h2f(L.k_rope_cache[(static_cast<size_t>(h) * max_len + pos) * rpad + (e - nope)]);
  if (e < hd) v = vbuf[static_cast<size_t>(pos) * H * hd + h * hd + e];
  const size_t o = (static_cast<size_t>(h) * max_len + pos) * kvpad + e;
  L.k_cache[o] = k;
  L.v_cache[o] = v;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

// Grid (ceil(count / 64), heads). DK: query/key dims (nope + rope) padded to 16 (= value dims padded).
// q from the entry rows (scaled by attn_scale, rope part rotated); keys and values from kv_split_kernel.
// Tiles of 64 positions are double-buffered with cp.async.
template <int DK>
__global__ void __launch_bounds__(kFaThreads, DK <= 64 ? 3 : 1) flash_attention_kernel(IvbLayerDesc L, const float* ent, int ld_ent,
                                                                     const __half* kh, const __half* kl,
                                                                     const __half* vh, const __half* vl, int Ppad,
                                                                     int start, int count, int d, int hd, int rope,
                                                                     int nope, float* y) {
  pdl_enter();
  constexpr int DV = DK;
  constexpr int kKs = DK + 8;       // key tile row stride (halves)
  constexpr int kVs = kFaPos + 8;   // transposed value tile row stride (halves)
  constexpr int kTileHalves = 2 * kFaPos * kKs + 2 * DV * kVs;  // k_hi, k_lo, v_hi, v_lo
  extern __shared__ __align__(16) unsigned char fa_smem[];
  __half* tiles = reinterpret_cast<__half*>(fa_smem);
  float* qs = reinterpret_cast<float*>(fa_smem);  // the query block, before the first key tile
  // grid (heads, query tiles) with the last query tile first: the causal tiles with the most keys start
  // in the first wave and the short ones fill the tail
  const int h = blockIdx.x, tq0 = (gridDim.y - 1 - blockIdx.y) * kFaTok;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, grp = lane >> 2, tig = lane & 3;
  const float scl = L.attn_scale;
  for (int i = tid; i < kFaTok * DK; i += kFaThreads) {
    const int tl = i / DK, e = i - tl * DK, t = tq0 + tl;
    float v = 0.0f;
    if (t < count && e < nope + rope) {
      const float* q = ent + static_cast<size_t>(t) * ld_ent + h * hd;
      if (e < nope) {
        v = q[e] * scl;
      } else {
        const int jr = (e - nope) >> 1;
        const float* rt = L.rope + static_cast<size_t>(start + t) * rope;
        const float cs = __ldg(rt + 2 * jr), sn = __ldg(rt + 2 * jr + 1);
        const float q0 = q[nope + 2 * jr], q1 = q[nope + 2 * jr + 1];
        v = (((e - nope) & 1) == 0 ? q0 * cs - q1 * sn : q0 * sn + q1 * cs) * scl;
      }
    }
    qs[i] = v;
  }
  __syncthreads();
  uint32_t qh[DK / 16][4], ql[DK / 16][4];
  const int r0 = 16 * warp + grp;
#pragma unroll
  for (int kk = 0; kk < DK / 16; ++kk) {
    const int c = 16 * kk + 2 * tig;
    split2(qs[r0 * DK + c], qs[r0 * DK + c + 1], qh[kk][0], ql[kk][0]);
    split2(qs[(r0 + 8) * DK + c], qs[(r0 + 8) * DK + c + 1], qh[kk][1], ql[kk][1]);
    split2(qs[r0 * DK + c + 8], qs[r0 * DK + c + 9], qh[kk][2], ql[kk][2]);
    split2(qs[(r0 + 8) * DK + c + 8], qs[(r0 + 8) * DK + c + 9], qh[kk][3], ql[kk][3]);
  }
  __syncthreads();  // qs is overwritten by the tiles
  const __half* khh = kh + static_cast<size_t>(h) * Ppad * DK;
  const __half* klh = kl + static_cast<size_t>(h) * Ppad * DK;
  const __half* vhh = vh + static_cast<size_t>(h) * DV * Ppad;
  const __half* vlh = vl + static_cast<size_t>(h) * DV * Ppad;
  auto load_tile = [&](int buf, int p0) {
    __half* base = tiles + buf * kTileHalves;
    __half* khs = base;
    __half* kls = khs + kFaPos * kKs;
    __half* vhs = kls + kFaPos * kKs;
    __half* vls = vhs + DV * kVs;
    for (int i = tid; i < kFaPos * (DK / 8); i += kFaThreads) {
      const int pl = i / (DK / 8), c = i - pl * (DK / 8);
      const size_t src = static_cast<size_t>(p0 + pl) * DK + 8 * c;
      cp_async16(khs + pl * kKs + 8 * c, khh + src);
      cp_async16(kls + pl * kKs + 8 * c, klh + src);
    }
    for (int i = tid; i < DV * (kFaPos / 8); i += kFaThreads) {
      const int e = i / (kFaPos / 8), c = i - e * (kFaPos / 8);
      const size_t src = static_cast<size_t>(e) * Ppad + p0 + 8 * c;
      cp_async16(vhs + e * kVs + 8 * c, vhh + src);
      cp_async16(vls + e * kVs + 8 * c, vlh + src);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  float o[DV / 8][4];
#pragma unroll
  for (int n = 0; n < DV / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
  const int pos_a = start + tq0 + r0, pos_b = pos_a + 8;  // positions of this thread's two query rows
  const int t_last = min(count, tq0 + kFaTok) - 1;
  const int p_end = start + t_last + 1;                   // keys 0..p_end-1 serve the block
  const int warp_last = start + min(count - 1, tq0 + 16 * warp + 15);
  const int tiles_n = (p_end + kFaPos - 1) / kFaPos;
  load_tile(0, 0);
  for (int it = 0; it < tiles_n; ++it) {
    const int p0 = it * kFaPos, buf = it & 1;
    if (it + 1 < tiles_n) {
      load_tile(buf ^ 1, p0 + kFaPos);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const __half* k_hi = tiles + buf * kTileHalves;
    const __half* k_lo = k_hi + kFaPos * kKs;
    const __half* v_hi = k_lo + kFaPos * kKs;
    const __half* v_lo = v_hi + DV * kVs;
    if (p0 <= warp_last) {
      float s[kFaPos / 8][4];
#pragma unroll
      for (int n = 0; n < kFaPos / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.0f;
      // the three products of a split go to one accumulator; consecutive MMAs target different
      // accumulators so none waits on the previous one
#pragma unroll
      for (int kk = 0; kk < DK / 16; ++kk) {
        uint32_t bh[kFaPos / 8][2], bl[kFaPos / 8][2];
#pragma unroll
        for (int n = 0; n < kFaPos / 8; ++n) {
          const int row = (8 * n + grp) * kKs + 16 * kk + 2 * tig;
          bh[n][0] = *reinterpret_cast<const uint32_t*>(k_hi + row);
          bh[n][1] = *reinterpret_cast<const uint32_t*>(k_hi + row + 8);
          bl[n][0] = *reinterpret_cast<const uint32_t*>(k_lo + row);
          bl[n][1] = *reinterpret_cast<const uint32_t*>(k_lo + row + 8);
        }
#pragma unroll
        for (int n = 0; n < kFaPos / 8; ++n) mma16816(s[n], qh[kk], bh[n][0], bh[n][1]);
#pragma unroll
        for (int n = 0; n < kFaPos / 8; ++n) mma16816(s[n], qh[kk], bl[n][0], bl[n][1]);
#pragma unroll
        for (int n = 0; n < kFaPos / 8; ++n) mma16816(s[n], ql[kk], bh[n][0], bh[n][1]);
      }
      // causal mask and online softmax (rows pos_a: s[n][0..1], pos_b: s[n][2..3])
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int n = 0; n < kFaPos / 8; ++n) {
        const int p = p0 + 8 * n + 2 * tig;
        if (p > pos_a) s[n][0] = -INFINITY;
        if (p + 1 > pos_a) s[n][1] = -INFINITY;
        if (p > pos_b) s[n][2] = -INFINITY;
        if (p + 1 > pos_b) s[n][3] = -INFINITY;
        mx[0] = fmaxf(mx[0], fmaxf(s[n][0], s[n][1]));
        mx[1] = fmaxf(mx[1], fmaxf(s[n][2], s[n][3]));
      }
      float corr[2], sum[2] = {0.0f, 0.0f};
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(kFull, mx[r], 1));
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(kFull, mx[r], 2));
        const float m_new = fmaxf(m_run[r], mx[r]);
        corr[r] = m_new == -INFINITY ? 1.0f : expf(m_run[r] - m_new);
        m_run[r] = m_new;
      }
      uint32_t ph[kFaPos / 16][4], pl2[kFaPos / 16][4];
#pragma unroll
      for (int n = 0; n < kFaPos / 8; ++n) {
        float e[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float m = m_run[c >> 1];
          e[c] = (s[n][c] == -INFINITY) ? 0.0f : expf(s[n][c] - m);
        }
        sum[0] += e[0] + e[1];
        sum[1] += e[2] + e[3];
        // C fragment of position tile n -> A fragment of k-step n / 2 (regs 0, 1 or 2, 3)
        split2(e[0], e[1], ph[n >> 1][(n & 1) * 2], pl2[n >> 1][(n & 1) * 2]);
        split2(e[2], e[3], ph[n >> 1][(n & 1) * 2 + 1], pl2[n >> 1][(n & 1) * 2 + 1]);
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        sum[r] += __shfl_xor_sync(kFull, sum[r], 1);
        sum[r] += __shfl_xor_sync(kFull, sum[r], 2);
        l_run[r] = l_run[r] * corr[r] + sum[r];
      }
#pragma unroll
      for (int n = 0; n < DV / 8; ++n) {
        o[n][0] *= corr[0];
        o[n][1] *= corr[0];
        o[n][2] *= corr[1];
        o[n][3] *= corr[1];
      }
#pragma unroll
      for (int kk = 0; kk < kFaPos / 16; ++kk) {
#pragma unroll
        for (int n0 = 0; n0 < DV / 8; n0 += 8) {  // eight value columns at a time bound the registers
          constexpr int kG = DV / 8 < 8 ? DV / 8 : 8;
          uint32_t bh[kG][2], bl[kG][2];
#pragma unroll
          for (int j = 0; j < kG; ++j) {
            const int row = (8 * (n0 + j) + grp) * kVs + 16 * kk + 2 * tig;
            bh[j][0] = *reinterpret_cast<const uint32_t*>(v_hi + row);
            bh[j][1] = *reinterpret_cast<const uint32_t*>(v_hi + row + 8);
            bl[j][0] = *reinterpret_cast<const uint32_t*>(v_lo + row);
            bl[j][1] = *reinterpret_cast<const uint32_t*>(v_lo + row + 8);
          }
#pragma unroll
          for (int j = 0; j < kG; ++j) mma16816(o[n0 + j], ph[kk], bh[j][0], bh[j][1]);
#pragma unroll
          for (int j = 0; j < kG; ++j) mma16816(o[n0 + j], ph[kk], bl[j][0], bl[j][1]);
#pragma unroll
          for (int j = 0; j < kG; ++j) mma16816(o[n0 + j], pl2[kk], bh[j][0], bh[j][1]);
        }
      }
    }
    __syncthreads();  // buffer buf is refilled by the next iteration's prefetch
  }
  const int ta = tq0 + r0, tb = ta + 8;
  const float inv_a = 1.0f / l_run[0], inv_b = 1.0f / l_run[1];
#pragma unroll
  for (int n = 0; n < DV / 8; ++n) {
    const int e = 8 * n + 2 * tig;
    if (ta < count) {
      if (e < hd) y[static_cast<size_t>(ta) * d + h * hd + e] = o[n][0] * inv_a;
      if (e + 1 < hd) y[static_cast<size_t>(ta) * d + h * hd + e + 1] = o[n][1] * inv_a;
    }
    if (tb < count) {
      if (e < hd) y[static_cast<size_t>(tb) * d + h * hd + e] = o[n][2] * inv_b;
      if (e + 1 < hd) y[static_cast<size_t>(tb) * d + h * hd + e + 1] = o[n][3] * inv_b;
    }
  }
}

template <int DK>
int32_t launch_fa(const IvbLayerDesc& L, const float* ent, int ld_ent, const float* knope, const float* vbuf,
                  __half* kvh, int start, int count, int d, int H, int hd, int rope, int nope, int max_len, int rpad,
                  float* y, cudaStream_t s) {
  const int P = start + count, Ppad = (P + kFaPos - 1) / kFaPos * kFaPos;
  const size_t per = static_cast<size_t>(H) * Ppad * DK;  // halves per split array
  __half *kh = kvh, *kl = kh + per, *vh = kl + per, *vl = vh + per;
  const int threads = H * Ppad * (DK / 8);
  IVB_CUDA(launch_pdl(kv_split_kernel<DK>, dim3((threads + 255) / 256), dim3(256), 0, s, L, knope, vbuf, P, Ppad, d, H, hd, rope, nope, max_len, rpad,
                                                            kh, kl, vh, vl));
  IVB_CUDA(cudaGetLastError());
  const size_t tile = (2 * static_cast<size_t>(kFaPos) * (DK + 8) + 2 * static_cast<size_t>(DK) * (kFaPos + 8)) * 2;
  const size_t smem = std::max(2 * tile, static_cast<size_t>(kFaTok) * DK * 4);
  IVB_CUDA(cudaFuncSetAttribute(flash_attention_kernel<DK>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  IVB_CUDA(launch_pdl(flash_attention_kernel<DK>, dim3(H, (count + kFaTok - 1) / kFaTok), dim3(kFaThreads), smem, s, 
      L, ent, ld_ent, kh, kl, vh, vl, Ppad, start, count, d, hd, rope, nope, y));
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

// Query/key dims (nope + rope) and value dims (head_dim) are equal for these models; both padded to 16.
int32_t launch_flash_attention(const IvbLayerDesc& L, const float* ent, int ld_ent, const float* knope, const float* vbuf,
                               __half* kvh, int start, int count, int d, int H, int hd, int rope, int nope, int max_len,
                               int rpad, float* y, cudaStream_t s) {
  const int dk = std::max(nope + rope, hd);
  if (dk <= 16) return launch_fa<16>(L, ent, ld_ent, knope, vbuf, kvh, start, count, d, H, hd, rope, nope, max_len, rpad, y, s);
  if (dk <= 32) return launch_fa<32>(L, ent, ld_ent, knope, vbuf, kvh, start, count, d, H, hd, rope, nope, max_len, rpad, y, s);
  if (dk <= 64) return launch_fa<64>(L, ent, ld_ent, knope, vbuf, kvh, start, count, d, H, hd, rope, nope, max_len, rpad, y, s);
  if (dk <= 128) return launch_fa<128>(L, ent, ld_ent, knope, vbuf, kvh, start, count, d, H, hd, rope, nope, max_len, rpad, y, s);
  return fail(IVB_EINVAL, "ivb_decoder_prefill: head dims %d beyond the attention kernel", dk);
}

__global__ void prefill_finish_kernel(const int64_t* tokens, int count, int pos_end, int64_t* token, int64_t* position) {
  pdl_enter();
  token[0] = tokens[count - 1];
  position[0] = pos_end;
}

struct PrefillLayout {
  size_t resid, ent, y, h, q8, scale, err, coef, cum, xend, carry, kvq8, knope, vbuf, kvh, partial, total;
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
  L.coef = take(T * md.heads * md.state_dim * 5 * 4);  // recurrence coefficients of a mamba block
  L.cum = take(T * md.heads * md.state_dim * 2 * 4);   // chunk-local decay products
  const size_t chunks = (T + kScanChunk - 1) / kScanChunk, lanes = static_cast<size_t>(md.heads) * md.state_dim * md.head_dim;
  L.xend = take(chunks * lanes * 2 * 4);                // chunk-end states of the zero-start scans
  L.carry = take(chunks * lanes * 2 * 4);               // chunk start states
  // latent attention: the cached latent of every position in the GEMM layout, and its keys and values
  bool mla = false;
  for (int i = 0; i < md.num_layers; ++i) mla = mla || layers[i].kind == IVB_MLA;
  const size_t P = mla ? static_cast<size_t>(md.max_len) : 0;
  L.kvq8 = take((P + 127) / 128 * 128 * ((md.latent_dim + 127) / 128 * 128));
  L.knope = take(P * md.heads * md.nope_dim * 4);
  L.vbuf = take(P * d * 4);
  const int dk_raw = std::max(md.nope_dim + md.rope_dim, md.head_dim);  // padded as launch_flash_attention does
  const size_t dk = dk_raw <= 16 ? 16 : dk_raw <= 32 ? 32 : dk_raw <= 64 ? 64 : 128;
  L.kvh = take(4 * static_cast<size_t>(md.heads) * ((P + 63) / 64 * 64) * dk * 2);
  L.partial = take(kGemmPartialFloats * 4);  // split-K partial sums of this call's GEMMs
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
  int8_t* kvq8 = reinterpret_cast<int8_t*>(ws + W.kvq8);
  float* knope = reinterpret_cast<float*>(ws + W.knope);
  float* vbuf = reinterpret_cast<float*>(ws + W.vbuf);
  __half* kvh = reinterpret_cast<__half*>(ws + W.kvh);
  float* partial = reinterpret_cast<float*>(ws + W.partial);
  float* coefb = reinterpret_cast<float*>(ws + W.coef);
  float* cumb = reinterpret_cast<float*>(ws + W.cum);
  float* xendb = reinterpret_cast<float*>(ws + W.xend);
  float* carryb = reinterpret_cast<float*>(ws + W.carry);
  int8_t* q8 = reinterpret_cast<int8_t*>(ws + W.q8);
  float* scale = reinterpret_cast<float*>(ws + W.scale);
  uint32_t* err = decoder_error_word(dec);  // reported by ivb_decoder_check
  if (err == nullptr) return fail(IVB_EINVAL, "ivb_decoder_prefill: bind the decoder first");
  const int lpad = static_cast<int>((Lt + 15) / 16 * 16), rpad = (rope + 7) / 8 * 8;
  IVB_CUDA(launch_pdl(embed_rows_kernel, dim3(count), dim3(kThreads), 0, s, md.head, tokens, d, resid));
  IVB_CUDA(cudaGetLastError());
  auto quant = [&](const float* x, int n, const float* norm, float eps) -> int32_t {
    const int ld = (n + 127) / 128 * 128;
    return ivb_quantize_rows(x, count, n, norm, eps, md.norm_clip, md.act_eps, q8, ld, scale, nullptr, stream);
  };
  auto gemm = [&](const IvbTernary& m, int epilogue, float* out, int ldo) -> int32_t {
    const int ld = (m.in_features + 127) / 128 * 128;
    return ternary_gemm_into(&m, q8, ld, scale, count, epilogue, out, ldo, err, partial, kGemmPartialFloats, stream);
  };
  for (int li = 0; li < md.num_layers; ++li) {
    const IvbLayerDesc& L = layers[li];
    if (int32_t rc = quant(resid, d, L.mixer_norm, L.mixer_norm_eps)) return rc;
    if (int32_t rc = gemm(L.entry, IVB_EPI_STORE, ent, L.entry.rows)) return rc;
    if (L.kind == IVB_MAMBA && hd >= 4) {
      const int ld = 2 * d + 3 * H * S;
      IVB_CUDA(launch_pdl(ssm_value_kernel, dim3((count * d + kThreads - 1) / kThreads), dim3(kThreads), 0, s, L, ent, count, d, ld, L.conv_taps, hbuf));
      IVB_CUDA(cudaGetLastError());
      IVB_CUDA(launch_pdl(ssm_coef_kernel, dim3((count * H * S + kThreads - 1) / kThreads), dim3(kThreads), 0, s, L, ent, count, d, H, S, ld, L.half_dt_min,
                                                                                 L.half_dt_range, coefb));
      IVB_CUDA(cudaGetLastError());
      const int nhc_max = std::min(H, (kScanCh - 1) / hd + 2);
      const size_t smem =
          (2 * (static_cast<size_t>(kScanBlock) * nhc_max * S * 5 + kScanBlock * kScanCh) + kScanBlock * kScanThreads) * 4;
      IVB_CUDA(cudaFuncSetAttribute(ssm_scan_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
      const int chunks = (count + kScanChunk - 1) / kScanChunk;
      IVB_CUDA(launch_pdl(ssm_cumprod_kernel, dim3((chunks * H * S + 127) / 128), dim3(128), 0, s, coefb, count, H, S, cumb));
      IVB_CUDA(cudaGetLastError());
      IVB_CUDA(launch_pdl(ssm_scan_block_kernel, dim3(dim3((d + kScanCh - 1) / kScanCh, chunks)), dim3(kScanThreads), smem, s, 
          L, ent, hbuf, coefb, count, d, H, hd, S, L.conv_taps, xendb, y));
      IVB_CUDA(cudaGetLastError());
      IVB_CUDA(launch_pdl(ssm_carry_kernel, dim3((H * S * hd + 127) / 128), dim3(128), 0, s, L, cumb, xendb, count, H, S, hd, carryb));
      IVB_CUDA(cudaGetLastError());
      IVB_CUDA(launch_pdl(ssm_output_kernel, dim3((count * d + kThreads - 1) / kThreads), dim3(kThreads), 0, s, L, ent, hbuf, coefb, cumb, carryb, count, d,
                                                                                  H, hd, S, y));
      IVB_CUDA(cudaGetLastError());
    } else if (L.kind == IVB_MAMBA) {
      const int blocks = (d * 16 + kThreads - 1) / kThreads;
      IVB_CUDA(launch_pdl(ssm_scan_kernel, dim3(blocks), dim3(kThreads), 0, s, L, ent, count, d, H, hd, S, L.conv_taps, L.half_dt_min, L.half_dt_range, y));
      IVB_CUDA(cudaGetLastError());
    } else {
      IVB_CUDA(launch_pdl(mla_cache_kernel, dim3(count), dim3(kThreads), 0, s, L, ent, start_position, d, Lt, H, rope, md.max_len, lpad, rpad, md.act_eps));
      IVB_CUDA(cudaGetLastError());
      // keys and values of positions 0..P-1 from the cached latent (earlier chunks included)
      const int P = start_position + count, ldl = (Lt + 127) / 128 * 128;
      const int chunks = P * (ldl >> 4);
      IVB_CUDA(launch_pdl(latent_tile_kernel, dim3((chunks + 255) / 256), dim3(256), 0, s, L.latent_q, lpad, Lt, P, ldl, kvq8));
      IVB_CUDA(cudaGetLastError());
      if (int32_t rc = ternary_gemm_into(&L.k_nope_up, kvq8, ldl, L.latent_scale, P, IVB_EPI_STORE, knope, H * nope, err, partial,
                                         kGemmPartialFloats, stream))
        return rc;
      if (int32_t rc = ternary_gemm_into(&L.v_up, kvq8, ldl, L.latent_scale, P, IVB_EPI_STORE, vbuf, d, err, partial,
                                         kGemmPartialFloats, stream))
        return rc;
      if (L.k_cache != nullptr && L.v_cache != nullptr) {  // the decode kernel's cache rows of the new positions
        const int kvpad = (hd + 3) & ~3;
        const long long n = static_cast<long long>(count) * H * kvpad;
        IVB_CUDA(launch_pdl(kv_cache_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, s, L, knope, vbuf,
                            start_position, count, H, hd, nope, md.max_len, rpad, kvpad));
        IVB_CUDA(cudaGetLastError());
      }
      if (int32_t rc = launch_flash_attention(L, ent, L.entry.rows, knope, vbuf, kvh, start_position, count, d, H, hd, rope,
                                              nope, md.max_len, rpad, y, s))
        return rc;
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
  IVB_CUDA(launch_pdl(prefill_finish_kernel, dim3(1), dim3(1), 0, s, tokens, count, start_position + count, md.token, md.position));
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

}  // extern "C"
