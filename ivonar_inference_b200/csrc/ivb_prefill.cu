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
#include "ivb_tc.cuh"
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

// ---- causal attention of the prefill ------------------------------------------------------------
// The reference decoder's form: the cached latent of every position p (int8 codes ql_p, scale a_p) is
// expanded by the tcgen05 GEMM into per-head keys K_nope[p] = a_p W_k ql_p + b_k and values V[p] =
// a_p W_v ql_p + b_v (the rows the decode kernel appends to its key/value cache). The attention itself
// runs on tcgen05 with fp16 operands in a three-product split (x = hi + lo, x.y ~ hi.hi' + hi.lo' +
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

// x = hi + lo with hi, lo fp16 (packed pairs)
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
  const __half l0 = __float2half_rn(x0 - __half2float(h0)), l1 = __float2half_rn(x1 - __half2float(h1));
  hi = static_cast<uint32_t>(__half_as_ushort(h0)) | (static_cast<uint32_t>(__half_as_ushort(h1)) << 16);
  lo = static_cast<uint32_t>(__half_as_ushort(l0)) | (static_cast<uint32_t>(__half_as_ushort(l1)) << 16);
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

// ---- causal prefill attention on the 5th-generation tensor cores ---------------------------------
// One CTA per (128 queries, head), 128 threads: thread r owns query row r, which is TMEM lane r of the
// two accumulators. Per tile of 64 keys: S = Q K^T and O_t = P V on tcgen05 (kind::f16, fp32 in TMEM),
// each as the three products of a hi/lo fp16 split (x = hi + lo; Qh Kh + Qh Kl + Ql Kh), issued by one
// thread and completed on an mbarrier by tcgen05.commit; between them each thread loads its score row
// from TMEM, masks it causally, runs the online softmax in registers and writes its probability row as
// the hi/lo A operand of P V. O accumulates in registers (o = o exp(m_old - m_new) + O_t). Every operand
// (Q, K, P, V) sits in shared memory as a K-major tile of 8-row x 16-byte core matrices (LBO 128 bytes);
// the key and value tiles come in that layout from fa_kv_tiles_kernel, one bulk copy each.
constexpr int kFaQ = 128;        // queries per CTA (MMA M, TMEM lanes)
constexpr int kFaKeys = 64;      // keys per tile (N of S, K of P V)
constexpr int kFaTcThreads = 128;

// Byte offset of 16-byte chunk c of row r in a K-major core-matrix tile with cpr chunks per row.
__host__ __device__ __forceinline__ int cm_off(int r, int c, int cpr) { return ((r >> 3) * cpr + c) * 128 + ((r & 7) << 4); }

// Keys and values of positions 0..P-1 of one layer as fp16 hi/lo tiles for the tensor-core attention:
// per (head, tile of 64 keys) a key tile [64 keys][DK dims] and a value tile [DK dims][64 keys], each a
// K-major core-matrix tile of DK * 64 halves; arrays kh, kl, vh, vl of H * Ppad * DK halves (Ppad = P
// rounded up to 64, padding zero). One thread per (head, position, 8 dims).
template <int DK>
__global__ void fa_kv_tiles_kernel(IvbLayerDesc L, const float* knope, const float* vbuf, int P, int Ppad, int d, int H, int hd,
                                   int rope, int nope, int max_len, int rpad, __half* kh, __half* kl, __half* vh, __half* vl) {
  pdl_enter();
  constexpr int cpr = DK / 8;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int per_head = Ppad * cpr;
  if (i >= H * per_head) return;
  const int h = i / per_head, rest = i - h * per_head, p = rest / cpr, c = rest - p * cpr;
  float kv[8], vv[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int e = 8 * c + j;
    float k = 0.0f, v = 0.0f;
    if (p < P) {
      if (e < nope) k = knope[static_cast<size_t>(p) * H * nope + h * nope + e];
      else if (e < nope + rope) k = h2f(L.k_rope_cache[(static_cast<size_t>(h) * max_len + p) * rpad + (e - nope)]);
      if (e < hd) v = vbuf[static_cast<size_t>(p) * d + h * hd + e];
    }
    kv[j] = k;
    vv[j] = v;
  }
  uint32_t khw[4], klw[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) split2(kv[2 * j], kv[2 * j + 1], khw[j], klw[j]);
  const size_t block = (static_cast<size_t>(h) * (Ppad / kFaKeys) + p / kFaKeys) * kFaKeys * DK * 2;  // bytes
  const int r = p & (kFaKeys - 1);
  unsigned char* khb = reinterpret_cast<unsigned char*>(kh) + block;
  unsigned char* klb = reinterpret_cast<unsigned char*>(kl) + block;
  *reinterpret_cast<uint4*>(khb + cm_off(r, c, cpr)) = make_uint4(khw[0], khw[1], khw[2], khw[3]);
  *reinterpret_cast<uint4*>(klb + cm_off(r, c, cpr)) = make_uint4(klw[0], klw[1], klw[2], klw[3]);
  // the value tile's rows are the dims: dim 8c + j of key r is half (r & 7) of chunk r / 8 of row 8c + j
  unsigned char* vhb = reinterpret_cast<unsigned char*>(vh) + block;
  unsigned char* vlb = reinterpret_cast<unsigned char*>(vl) + block;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const __half hv = __float2half_rn(vv[j]);
    const int off = cm_off(8 * c + j, r >> 3, kFaKeys / 8) + (r & 7) * 2;
    *reinterpret_cast<__half*>(vhb + off) = hv;
    *reinterpret_cast<__half*>(vlb + off) = __float2half_rn(vv[j] - __half2float(hv));
  }
}

// Grid (heads, query blocks of 128, last block first). q from the entry rows (scaled by attn_scale, rope
// pairs rotated), keys and values from fa_kv_tiles_kernel; y [count][d] gets the head's outputs. Every
// wait is bounded: a wait that runs out records IVB_ETIMEOUT in *error and the CTA stops after the
// tensor-core work it issued has completed (bounded again), releasing its tensor memory.
template <int DK>
__global__ void __launch_bounds__(kFaTcThreads, 1)
    flash_attention_tc_kernel(IvbLayerDesc L, const float* ent, int ld_ent, const __half* kh, const __half* kl, const __half* vh,
                              const __half* vl, int Ppad, int start, int count, int d, int hd, int rope, int nope, float* y,
                              unsigned long long timeout_ns, unsigned* error) {
  pdl_enter();
  constexpr int cq = DK / 8;                        // 16-byte chunks per query / key row
  constexpr int kQBytes = kFaQ * DK * 2;            // one of Qh, Ql
  constexpr int kKBytes = kFaKeys * DK * 2;         // one of Kh, Kl, Vh, Vl
  constexpr int kPBytes = kFaQ * kFaKeys * 2;       // one of Ph, Pl
  constexpr int kTmemCols = (kFaKeys + DK) <= 128 ? 128 : 256;
  constexpr uint32_t kIdescS = idesc_f16(kFaQ, kFaKeys), kIdescO = idesc_f16(kFaQ, DK);
  extern __shared__ __align__(128) unsigned char fa_tc_smem[];
  unsigned char* const qhs = fa_tc_smem;
  unsigned char* const qls = qhs + kQBytes;
  unsigned char* const khs = qls + kQBytes;
  unsigned char* const kls = khs + kKBytes;
  unsigned char* const vhs = kls + kKBytes;
  unsigned char* const vls = vhs + kKBytes;
  unsigned char* const phs = vls + kKBytes;
  unsigned char* const pls = phs + kPBytes;
  __shared__ __align__(8) unsigned long long kbar, vbar, sbar, obar;
  __shared__ unsigned tmem_base;
  const int h = blockIdx.x, tq0 = (gridDim.y - 1 - blockIdx.y) * kFaQ;
  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid == 0) {
    mbar_init(&kbar, 1);
    mbar_init(&vbar, 1);
    mbar_init(&sbar, 1);
    mbar_init(&obar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // my query row (scaled, rope pairs rotated) as hi/lo fp16 chunks of the A operand of S
  const int t = tq0 + tid;
  {
    const float scl = L.attn_scale;
    const float* q = ent + static_cast<size_t>(t < count ? t : 0) * ld_ent + h * hd;
    const float* rt = L.rope + static_cast<size_t>(start + (t < count ? t : 0)) * rope;
#pragma unroll
    for (int c = 0; c < cq; ++c) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int e = 8 * c + j;
        float x = 0.0f;
        if (t < count && e < nope + rope) {
          if (e < nope) {
            x = q[e] * scl;
          } else {
            const int jr = (e - nope) >> 1;
            const float cs = __ldg(rt + 2 * jr), sn = __ldg(rt + 2 * jr + 1);
            const float q0 = q[nope + 2 * jr], q1 = q[nope + 2 * jr + 1];
            x = (((e - nope) & 1) == 0 ? q0 * cs - q1 * sn : q0 * sn + q1 * cs) * scl;
          }
        }
        v[j] = x;
      }
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) split2(v[2 * j], v[2 * j + 1], hw[j], lw[j]);
      *reinterpret_cast<uint4*>(qhs + cm_off(tid, c, cq)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(qls + cm_off(tid, c, cq)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the MMA reads what the threads wrote
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = tmem_base;
  const unsigned tS = tmem, tO = tmem + kFaKeys;  // S in columns [0, 64), O_t in [64, 64 + DK)
  const unsigned lane_off = static_cast<unsigned>(32 * warp) << 16;
  const int t_last = min(count, tq0 + kFaQ) - 1;
  const int p_end = start + t_last + 1;  // keys 0..p_end-1 serve the block
  const int tiles_n = (p_end + kFaKeys - 1) / kFaKeys;
  const int pos = start + t;            // my query's position
  const size_t head_tiles = static_cast<size_t>(Ppad / kFaKeys);
  float o[DK];
#pragma unroll
  for (int e = 0; e < DK; ++e) o[e] = 0.0f;
  float m_run = -INFINITY, l_run = 0.0f;
  // Pipeline (thread 0 issues; every thread runs the softmax): the key tile of it + 1 is copied as soon
  // as S(it) is done with the key buffer, the value tile of it + 1 as soon as O(it) is done with the
  // value buffer, and S(it + 1) is issued right behind O(it), so the tensor pipe runs O(it) and S(it + 1)
  // while the threads take O(it) out of TMEM. Thread 0 keeps the parity of every copy and commit it
  // issued and has not waited for (-1: none), to drain them if a wait runs out.
  int k_pend = -1, v_pend = -1, s_pend = -1, o_pend = -1;
  const unsigned char* const khg = reinterpret_cast<const unsigned char*>(kh) + static_cast<size_t>(h) * head_tiles * kKBytes;
  const unsigned char* const klg = reinterpret_cast<const unsigned char*>(kl) + static_cast<size_t>(h) * head_tiles * kKBytes;
  const unsigned char* const vhg = reinterpret_cast<const unsigned char*>(vh) + static_cast<size_t>(h) * head_tiles * kKBytes;
  const unsigned char* const vlg = reinterpret_cast<const unsigned char*>(vl) + static_cast<size_t>(h) * head_tiles * kKBytes;
  auto issue_k = [&](int it) {
    mbar_expect_tx(&kbar, 2u * kKBytes);
    bulk_copy(khs, khg + static_cast<size_t>(it) * kKBytes, kKBytes, &kbar);
    bulk_copy(kls, klg + static_cast<size_t>(it) * kKBytes, kKBytes, &kbar);
    k_pend = it & 1;
  };
  auto issue_v = [&](int it) {
    mbar_expect_tx(&vbar, 2u * kKBytes);
    bulk_copy(vhs, vhg + static_cast<size_t>(it) * kKBytes, kKBytes, &vbar);
    bulk_copy(vls, vlg + static_cast<size_t>(it) * kKBytes, kKBytes, &vbar);
    v_pend = it & 1;
  };
  const unsigned qa = smem_addr(qhs), qb = smem_addr(qls), ka = smem_addr(khs), kb = smem_addr(kls);
  const unsigned pa = smem_addr(phs), pb = smem_addr(pls), va = smem_addr(vhs), vb = smem_addr(vls);
  auto issue_s = [&](int it) {  // S = Q K^T
    tc_fence_after();
#pragma unroll
    for (int kk = 0; kk < DK / 16; ++kk) {
      const unsigned off = kk * 256;
      umma_f16_ss(tS, smem_desc(qa + off, cq * 128), smem_desc(ka + off, cq * 128), kIdescS, kk > 0);
      umma_f16_ss(tS, smem_desc(qa + off, cq * 128), smem_desc(kb + off, cq * 128), kIdescS, true);
      umma_f16_ss(tS, smem_desc(qb + off, cq * 128), smem_desc(ka + off, cq * 128), kIdescS, true);
    }
    umma_commit(&sbar);
    s_pend = it & 1;
  };
  auto issue_o = [&](int it) {  // O_t = P V
    tc_fence_after();
#pragma unroll
    for (int kk = 0; kk < kFaKeys / 16; ++kk) {
      const unsigned off = kk * 256;
      umma_f16_ss(tO, smem_desc(pa + off), smem_desc(va + off), kIdescO, kk > 0);
      umma_f16_ss(tO, smem_desc(pa + off), smem_desc(vb + off), kIdescO, true);
      umma_f16_ss(tO, smem_desc(pb + off), smem_desc(va + off), kIdescO, true);
    }
    umma_commit(&obar);
    o_pend = it & 1;
  };
  bool t0_ok = true;  // thread 0's own waits (the key and value copies)
  if (tid == 0) {
    issue_k(0);
    issue_v(0);
    t0_ok = mbar_wait_bounded(&kbar, 0u, timeout_ns);
    if (t0_ok) {
      k_pend = -1;
      issue_s(0);
    }
  }
  bool ok = true;
  constexpr float kLog2e = 1.4426950408889634f;
  for (int it = 0; it < tiles_n; ++it) {
    const unsigned par = static_cast<unsigned>(it) & 1u;
    if (__syncthreads_or((tid == 0 && !t0_ok) || !mbar_wait_bounded(&sbar, par, timeout_ns))) {
      ok = false;
      break;
    }
    tc_fence_after();
    if (tid == 0) {
      s_pend = -1;
      if (it + 1 < tiles_n) issue_k(it + 1);  // S(it) is done with the key buffer
    }
    // my score row, causally masked; online softmax (exp2 of log2e-scaled differences); probabilities
    // as the hi/lo A operand of P V (the previous P V finished with it)
    const int p0 = it * kFaKeys;
    float sc[kFaKeys];
    {
      uint32_t v[32];
      tmem_ld32(tS + lane_off, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) sc[j] = __uint_as_float(v[j]);
      tmem_ld32(tS + lane_off + 32, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) sc[32 + j] = __uint_as_float(v[j]);
    }
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kFaKeys; ++j) {
      if (p0 + j > pos) sc[j] = -INFINITY;
      mx = fmaxf(mx, sc[j]);
    }
    const float m_new = fmaxf(m_run, mx);
    const float corr = m_new == -INFINITY ? 1.0f : exp2f((m_run - m_new) * kLog2e);
    const float mb = m_new == -INFINITY ? 0.0f : m_new * kLog2e;
    float sum = 0.0f;
#pragma unroll
    for (int c = 0; c < kFaKeys / 8; ++c) {
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float e0 = exp2f(fmaf(sc[8 * c + 2 * j], kLog2e, -mb));
        const float e1 = exp2f(fmaf(sc[8 * c + 2 * j + 1], kLog2e, -mb));
        sum += e0 + e1;
        split2(e0, e1, hw[j], lw[j]);
      }
      *reinterpret_cast<uint4*>(phs + cm_off(tid, c, kFaKeys / 8)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(pls + cm_off(tid, c, kFaKeys / 8)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
    l_run = l_run * corr + sum;
    m_run = m_new;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();  // P(it) written; every thread has read S(it)
    if (tid == 0 && t0_ok) {
      t0_ok = mbar_wait_bounded(&vbar, par, timeout_ns);  // V(it)
      if (t0_ok) {
        v_pend = -1;
        issue_o(it);
        if (it + 1 < tiles_n) {
          t0_ok = mbar_wait_bounded(&kbar, (par ^ 1u), timeout_ns);  // K(it + 1)
          if (t0_ok) {
            k_pend = -1;
            issue_s(it + 1);
          }
        }
      }
    }
    if (__syncthreads_or((tid == 0 && !t0_ok) || !mbar_wait_bounded(&obar, par, timeout_ns))) {
      ok = false;
      break;
    }
    tc_fence_after();
    if (tid == 0) {
      o_pend = -1;
      if (it + 1 < tiles_n) issue_v(it + 1);  // O(it) is done with the value buffer
    }
#pragma unroll
    for (int c0 = 0; c0 < DK; c0 += 16) {
      uint32_t v[16];
      tmem_ld16(tO + lane_off + c0, v);
#pragma unroll
      for (int j = 0; j < 16; ++j) o[c0 + j] = fmaf(o[c0 + j], corr, __uint_as_float(v[j]));
    }
    tc_fence_before();
    __syncthreads();  // every thread has read O(it) before O(it + 1) is issued
  }
  if (!ok) {
    if (tid == 0) {
      atomicCAS(error, 0u, static_cast<unsigned>(IVB_ETIMEOUT));
      // let the copies and the tensor-core work this CTA issued finish before its shared and tensor
      // memory are released
      if (k_pend >= 0) mbar_wait_bounded(&kbar, static_cast<unsigned>(k_pend), timeout_ns);
      if (v_pend >= 0) mbar_wait_bounded(&vbar, static_cast<unsigned>(v_pend), timeout_ns);
      if (s_pend >= 0) mbar_wait_bounded(&sbar, static_cast<unsigned>(s_pend), timeout_ns);
      if (o_pend >= 0) mbar_wait_bounded(&obar, static_cast<unsigned>(o_pend), timeout_ns);
    }
  } else if (t < count) {
    const float inv = 1.0f / l_run;
    float* yr = y + static_cast<size_t>(t) * d + h * hd;
#pragma unroll
    for (int e = 0; e < DK; ++e)
      if (e < hd) yr[e] = o[e] * inv;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

template <int DK>
int32_t launch_fa(const IvbLayerDesc& L, const float* ent, int ld_ent, const float* knope, const float* vbuf,
                  __half* kvh, int start, int count, int d, int H, int hd, int rope, int nope, int max_len, int rpad,
                  float* y, unsigned* error, cudaStream_t s) {
  const int P = start + count, Ppad = (P + kFaKeys - 1) / kFaKeys * kFaKeys;
  const size_t per = static_cast<size_t>(H) * Ppad * DK;  // halves per split array
  __half *kh = kvh, *kl = kh + per, *vh = kl + per, *vl = vh + per;
  const int threads = H * Ppad * (DK / 8);
  IVB_CUDA(launch_pdl(fa_kv_tiles_kernel<DK>, dim3((threads + 255) / 256), dim3(256), 0, s, L, knope, vbuf, P, Ppad, d, H, hd, rope,
                      nope, max_len, rpad, kh, kl, vh, vl));
  IVB_CUDA(cudaGetLastError());
  const size_t smem = 2 * static_cast<size_t>(kFaQ) * DK * 2 + 4 * static_cast<size_t>(kFaKeys) * DK * 2 + 2 * static_cast<size_t>(kFaQ) * kFaKeys * 2;
  IVB_CUDA(cudaFuncSetAttribute(flash_attention_tc_kernel<DK>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  IVB_CUDA(launch_pdl(flash_attention_tc_kernel<DK>, dim3(H, (count + kFaQ - 1) / kFaQ), dim3(kFaTcThreads), smem, s, L, ent, ld_ent, kh,
                      kl, vh, vl, Ppad, start, count, d, hd, rope, nope, y, 2000000000ull, error));
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

// Query/key dims (nope + rope) and value dims (head_dim) are equal for these models; both padded to 16.
int32_t launch_flash_attention(const IvbLayerDesc& L, const float* ent, int ld_ent, const float* knope, const float* vbuf,
                               __half* kvh, int start, int count, int d, int H, int hd, int rope, int nope, int max_len,
                               int rpad, float* y, unsigned* error, cudaStream_t s) {
  const int dk = std::max(nope + rope, hd);
  if (dk <= 16) return launch_fa<16>(L, ent, ld_ent, knope, vbuf, kvh, start, count, d, H, hd, rope, nope, max_len, rpad, y, error, s);
  if (dk <= 32) return launch_fa<32>(L, ent, ld_ent, knope, vbuf, kvh, start, count, d, H, hd, rope, nope, max_len, rpad, y, error, s);
  if (dk <= 64) return launch_fa<64>(L, ent, ld_ent, knope, vbuf, kvh, start, count, d, H, hd, rope, nope, max_len, rpad, y, error, s);
  if (dk <= 128) return launch_fa<128>(L, ent, ld_ent, knope, vbuf, kvh, start, count, d, H, hd, rope, nope, max_len, rpad, y, error, s);
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
                                              nope, md.max_len, rpad, y, err, s))
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
