// Device building blocks of the sm_100a Ivonar token loop.
//
// Every block here runs with kThreads = 256 threads per CTA. The same functions
// serve the single-launch unit entry points (ivb_unit.cu) and the persistent
// multi-layer decode kernel (ivb_decoder.cu), so the unit parity tests exercise
// the production arithmetic.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#include "ivonar_b200.h"

namespace ivb {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kPrefetch = 8;          // weight chunks (16 B) per thread held in registers across a barrier
constexpr int kMaxLatentPerLane = 16;  // latent_dim <= 512
constexpr int kMaxStateDim = 16;
constexpr int kMaxTopK = 1024;
constexpr unsigned kFull = 0xffffffffu;

// ------------------------------------------------------------------------------------------------
// small helpers
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ float ldcg_f(const float* p) { return __ldcg(p); }
__device__ __forceinline__ long long ldcg_i64(const int64_t* p) {
  return __ldcg(reinterpret_cast<const long long*>(p));
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// Canonical block sum: per-warp xor butterfly (offsets 16..1), then warps 0..7 added in order.
// The CPU oracle restates this order exactly, which makes the quantised codes bit-identical.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFull, v, off);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, off));
  return v;
}
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = red[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) t += red[w];
  __syncthreads();
  return t;
}
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = red[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) t = fmaxf(t, red[w]);
  __syncthreads();
  return t;
}

// ------------------------------------------------------------------------------------------------
// Activation layout in shared memory.
// A 16-byte weight chunk u holds inputs 64u..64u+63: word k (bytes 4k..4k+3) holds inputs
// 64u+16k+4c+f in bits 2f of byte c. One dp4a over (word >> 2f) & 0x03030303 needs the four
// activations 64u+16k+f+{0,4,8,12} packed in one int, so the codes are stored transposed inside
// each 16-input block, and the four 16-byte blocks of a chunk are rotated by (u>>1)&3 so that the
// 128-bit shared loads of eight consecutive chunks hit eight distinct bank groups.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ int act_slot(int i) {
  const int u = i >> 6, k = (i >> 4) & 3;
  const int slot = (k + ((u >> 1) & 3)) & 3;
  return (u << 6) + (slot << 4) + ((i & 3) << 2) + ((i >> 2) & 3);
}

// int32 sum over 64 inputs of code * q8 (codes 0..2 = ternary value + 1).
__device__ __forceinline__ int chunk_dot(const uint4 w, const int8_t* act, int u) {
  const int rot = (u >> 1) & 3;
  const char* base = reinterpret_cast<const char*>(act) + (u << 6);
  const int4 a0 = *reinterpret_cast<const int4*>(base + (((0 + rot) & 3) << 4));
  const int4 a1 = *reinterpret_cast<const int4*>(base + (((1 + rot) & 3) << 4));
  const int4 a2 = *reinterpret_cast<const int4*>(base + (((2 + rot) & 3) << 4));
  const int4 a3 = *reinterpret_cast<const int4*>(base + (((3 + rot) & 3) << 4));
  int d = 0;
  d = __dp4a(static_cast<int>(w.x & 0x03030303u), a0.x, d);
  d = __dp4a(static_cast<int>((w.x >> 2) & 0x03030303u), a0.y, d);
  d = __dp4a(static_cast<int>((w.x >> 4) & 0x03030303u), a0.z, d);
  d = __dp4a(static_cast<int>((w.x >> 6) & 0x03030303u), a0.w, d);
  d = __dp4a(static_cast<int>(w.y & 0x03030303u), a1.x, d);
  d = __dp4a(static_cast<int>((w.y >> 2) & 0x03030303u), a1.y, d);
  d = __dp4a(static_cast<int>((w.y >> 4) & 0x03030303u), a1.z, d);
  d = __dp4a(static_cast<int>((w.y >> 6) & 0x03030303u), a1.w, d);
  d = __dp4a(static_cast<int>(w.z & 0x03030303u), a2.x, d);
  d = __dp4a(static_cast<int>((w.z >> 2) & 0x03030303u), a2.y, d);
  d = __dp4a(static_cast<int>((w.z >> 4) & 0x03030303u), a2.z, d);
  d = __dp4a(static_cast<int>((w.z >> 6) & 0x03030303u), a2.w, d);
  d = __dp4a(static_cast<int>(w.w & 0x03030303u), a3.x, d);
  d = __dp4a(static_cast<int>((w.w >> 2) & 0x03030303u), a3.y, d);
  d = __dp4a(static_cast<int>((w.w >> 4) & 0x03030303u), a3.z, d);
  d = __dp4a(static_cast<int>((w.w >> 6) & 0x03030303u), a3.w, d);
  return d;
}

// ------------------------------------------------------------------------------------------------
// Canonical per-token int8 quantiser (optionally with RMSNorm: clamp(x * inv_rms, +-clip) * w).
// xv holds the fp32 input (n values, shared). Thread t owns inputs t, t+256, ...; the sum of squares
// uses fmaf in that order, then block_sum. inv_rms = 1 / sqrtf(ss / n + eps) (IEEE sqrt and divide),
// scale = max(amax / 127, act_eps), code = rintf(v / scale). Writes codes either in the transposed
// GEMV layout (transposed = true) or in natural order, and 64-input chunk sums to xsum (if given).
// Returns the activation scale. Reference: ternary.cu:148-197, cpu_decoder.py:30-70.
// ------------------------------------------------------------------------------------------------
static __device__ float quantize_block(float* xv, int n, const float* norm_w, float norm_eps, float clip, float act_eps,
                                int8_t* codes, bool transposed, int* xsum, float* red) {
  const int tid = threadIdx.x;
  const int chunks = (n + 63) >> 6;
  if (norm_w != nullptr) {
    float p = 0.0f;
    for (int i = tid; i < n; i += kThreads) {
      const float x = xv[i];
      p = fmaf(x, x, p);
    }
    const float ss = block_sum(p, red);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(n) + norm_eps);
    for (int i = tid; i < n; i += kThreads) {
      const float a = __fmul_rn(xv[i], inv);
      xv[i] = __fmul_rn(fminf(fmaxf(a, -clip), clip), __ldg(norm_w + i));
    }
  }
  float am = 0.0f;
  for (int i = tid; i < n; i += kThreads) am = fmaxf(am, fabsf(xv[i]));
  const float amax = block_max(am, red);
  const float scale = fmaxf(amax / 127.0f, act_eps);
  for (int i = tid; i < n; i += kThreads) {
    const int q = static_cast<int>(rintf(xv[i] / scale));
    codes[transposed ? act_slot(i) : i] = static_cast<int8_t>(q);
  }
  for (int i = n + tid; i < (chunks << 6); i += kThreads) codes[transposed ? act_slot(i) : i] = 0;
  __syncthreads();
  if (xsum != nullptr) {
    for (int u = tid; u < chunks; u += kThreads) {
      const int* words = reinterpret_cast<const int*>(codes + (u << 6));
      int total = 0;
#pragma unroll
      for (int w = 0; w < 16; ++w) total = __dp4a(words[w], 0x01010101, total);
      xsum[u] = total;
    }
    __syncthreads();
  }
  return scale;
}

// ------------------------------------------------------------------------------------------------
// GEMV phase: one CTA computes rows [r0, r1) of a ternary matrix against the quantised input.
// Lanes per row (lpr, power of two <= 32) walk the 16-byte chunks of a row; rpi = 256/lpr rows per
// iteration. A thread's work items q = it * kpl + j (row iteration it, chunk j) are streamed through
// a kPrefetch-deep register ring, so the first kPrefetch chunks can be loaded before the CTA waits
// for the input vector.
// ------------------------------------------------------------------------------------------------
struct GemvGeom {
  int r0, r1;       // CTA row range
  int lpr_log;      // log2 lanes per row
  int kpl;          // chunks per lane per row
  int chunks;       // chunks per row
  int iters;        // row iterations
};

__device__ __forceinline__ GemvGeom gemv_geom(const IvbTernary& m, int rows_per_cta, int lpr_log, int cta) {
  GemvGeom g;
  g.r0 = min(m.rows, cta * rows_per_cta);
  g.r1 = min(m.rows, g.r0 + rows_per_cta);
  g.lpr_log = lpr_log;
  g.chunks = (m.in_features + 63) >> 6;
  g.kpl = (g.chunks + (1 << lpr_log) - 1) >> lpr_log;
  const int rpi = kThreads >> lpr_log;
  g.iters = (g.r1 - g.r0 + rpi - 1) / rpi;
  return g;
}

__device__ __forceinline__ void gemv_item(const IvbTernary& m, const GemvGeom& g, int q, int& row, int& u, bool& valid) {
  const int it = q / g.kpl, j = q - it * g.kpl;
  const int tid = threadIdx.x;
  row = g.r0 + it * (kThreads >> g.lpr_log) + (tid >> g.lpr_log);
  u = (tid & ((1 << g.lpr_log) - 1)) + (j << g.lpr_log);
  valid = row < g.r1 && u < g.chunks;
}

__device__ __forceinline__ void gemv_load(const IvbTernary& m, int row, int u, bool valid, uint4& w, float& s) {
  if (valid) {
    w = __ldg(reinterpret_cast<const uint4*>(m.packed + static_cast<size_t>(row) * m.row_bytes) + u);
    s = h2f(__ldg(m.scales + static_cast<size_t>(row) * m.scale_stride + (u >> 1)));
  } else {
    w = make_uint4(0u, 0u, 0u, 0u);
    s = 0.0f;
  }
}

__device__ __forceinline__ void gemv_prefetch(const IvbTernary& m, const GemvGeom& g, uint4 (&pf)[kPrefetch],
                                              float (&pfs)[kPrefetch]) {
  const int nq = g.iters * g.kpl;
#pragma unroll
  for (int s = 0; s < kPrefetch; ++s) {
    int row, u;
    bool valid;
    gemv_item(m, g, s, row, u, valid);
    gemv_load(m, row, u, valid && s < nq, pf[s], pfs[s]);
  }
}

// Dot products, reduction across lanes and epilogue. act/xsum/scale come from quantize_block.
// res: shared scratch of kThreads floats (silu pairing).
static __device__ void gemv_rows(const IvbTernary& m, const GemvGeom& g, const int8_t* act, const int* xsum, float act_scale,
                          int epilogue, float* out, uint4 (&pf)[kPrefetch], float (&pfs)[kPrefetch], float* res) {
  const int tid = threadIdx.x;
  const int lpr = 1 << g.lpr_log;
  const int rpi = kThreads >> g.lpr_log;
  const int nq = g.iters * g.kpl;
  float acc = 0.0f;
  for (int q0 = 0; q0 < nq; q0 += kPrefetch) {
#pragma unroll
    for (int s = 0; s < kPrefetch; ++s) {
      const int q = q0 + s;
      if (q < nq) {
        const uint4 w = pf[s];
        const float sc = pfs[s];
        int row, u;
        bool valid;
        gemv_item(m, g, q, row, u, valid);
        {
          int nrow, nu;
          bool nvalid;
          gemv_item(m, g, q + kPrefetch, nrow, nu, nvalid);
          gemv_load(m, nrow, nu, nvalid && q + kPrefetch < nq, pf[s], pfs[s]);
        }
        if (valid) {
          const int d = chunk_dot(w, act, u) - xsum[u];
          acc = fmaf(static_cast<float>(d), sc, acc);
        }
        const int it = q / g.kpl;
        if (q - it * g.kpl == g.kpl - 1) {
          // row end (uniform across the CTA): reduce over the lpr lanes of this row
          for (int off = 1; off < lpr; off <<= 1) acc += __shfl_xor_sync(kFull, acc, off);
          const int r = g.r0 + it * rpi + (tid >> g.lpr_log);
          float result = acc * act_scale;
          const bool lead = (tid & (lpr - 1)) == 0 && r < g.r1;
          if (lead && m.bias != nullptr) result += __ldg(m.bias + r);
          if (epilogue == IVB_EPI_SILU_PAIR) {
            if ((tid & (lpr - 1)) == 0) res[tid >> g.lpr_log] = result;
            __syncthreads();
            const int slot = tid;
            if (slot < rpi && (slot & 1) == 0) {
              const int rr = g.r0 + it * rpi + slot;
              if (rr + 1 < g.r1 + 1 && rr < g.r1) out[rr >> 1] = silu_f(res[slot]) * res[slot + 1];
            }
            __syncthreads();
          } else if (lead) {
            if (epilogue == IVB_EPI_RESIDUAL) out[r] = ldcg_f(out + r) + result;
            else out[r] = result;
          }
          acc = 0.0f;
        }
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Recurrent (SSM) step for channels [c0, c1). 16 threads per channel, one per state index.
// Reference: ternary.cu:421-482, cpu_decoder.py:137-183, decoder.py:235-264.
// mixer_in = [value (hidden) | gate (hidden) | bc_dt (heads * 3 * state)].
// ------------------------------------------------------------------------------------------------
static __device__ void ssm_channels(const IvbLayerDesc& L, int hidden, int heads, int head_dim, int state_dim,
                             const float* mixer_in, float* y, int c0, int c1) {
  const int tid = threadIdx.x;
  const int s = tid & 15, slot = tid >> 4;
  const int taps = L.conv_taps;
  for (int cb = c0; cb < c1; cb += kThreads / 16) {
    const int c = cb + slot;
    const bool live = c < c1;
    float value = 0.0f;
    if (live && s == 0) {
      const float* w = L.conv_weight + static_cast<size_t>(c) * taps;
      float* win = L.conv_state + static_cast<size_t>(c) * (taps - 1);
      const float incoming = ldcg_f(mixer_in + c);
      float conv = __ldg(L.conv_bias + c);
      for (int k = 0; k < taps - 1; ++k) conv = fmaf(__ldg(w + k), win[k], conv);
      conv = fmaf(__ldg(w + taps - 1), incoming, conv);
      for (int k = 0; k + 1 < taps - 1; ++k) win[k] = win[k + 1];
      if (taps > 1) win[taps - 2] = incoming;
      value = silu_f(conv);
    }
    value = __shfl_sync(kFull, value, (threadIdx.x & 31) & ~15);
    float contrib = 0.0f;
    if (live && s < state_dim) {
      const int h = c / head_dim, d = c - h * head_dim;
      const float* bcdt = mixer_in + 2 * hidden + h * 3 * state_dim;
      const float b = tanhf(ldcg_f(bcdt + s));
      const float cc = tanhf(ldcg_f(bcdt + state_dim + s));
      const float half_dt = L.half_dt_min + sigmoid_f(ldcg_f(bcdt + 2 * state_dim + s)) * L.half_dt_range;
      const int hs = h * state_dim + s;
      const float mag = expf(2.0f * half_dt * __ldg(L.decay + hs));
      float sn, cs;
      sincosf(2.0f * half_dt * __ldg(L.theta + hs), &sn, &cs);
      const float ar = mag * cs, ai = mag * sn;
      const size_t idx = static_cast<size_t>(hs) * head_dim + d;
      const float prev = L.prev_force[idx];
      float* st = L.ssm_state + 2 * idx;
      const float sr = st[0], si = st[1];
      const float force = b * value;
      const float dr = (force + ar * prev) * half_dt;
      const float di = (ai * prev) * half_dt;
      const float nr = sr * ar - si * ai + dr;
      const float ni = sr * ai + si * ar + di;
      st[0] = nr;
      st[1] = ni;
      L.prev_force[idx] = force;
      contrib = cc * nr;
    }
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) contrib += __shfl_xor_sync(kFull, contrib, off);
    if (live && s == 0) {
      const float gate = ldcg_f(mixer_in + hidden + c);
      y[c] = (contrib + __ldg(L.skip + c) * value) * sigmoid_f(gate);
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Latent attention for one head over the compressed cache (absorbed up-projections).
//   score_t = a_t * <qa, ql_t> + qb + <q_rope_rot, k_rope_rot_t>     (qa = s * q_nope^T W_knope_h)
//   out_h   = W_v_h (sum_t p_t a_t ql_t) + b_v_h
// Exactly the reference's softmax(q.k) v with k_nope = up(latent), v = up(latent) (linear in the
// int8 latent codes); reference ternary.cu:509-611, decoder.py:271-297, attention.py:136-151.
// mixer_in = [q (hidden) | latent (L) | k_rope (heads * rope)].
// ------------------------------------------------------------------------------------------------
struct AttnSmem {
  float* xv;      // [L]   latent fp32 (quantiser input)
  int8_t* ql;     // [L]   codes of the current latent
  float* qa;      // [L]
  float* qr;      // [rope]  rotated, scaled query rope part
  float* kr;      // [rope]  rotated k_rope of the current position
  float* qn;      // [nope]  scaled query nope part
  float* part;    // [kWarps][L + 2]
  float* red;     // [64]
};

__device__ __forceinline__ float ternary_code_value(const uint8_t* row, int j) {
  return static_cast<float>(static_cast<int>((__ldg(row + (j >> 2)) >> ((j & 3) << 1)) & 3) - 1);
}

static __device__ void attention_head(const IvbLayerDesc& L, int hidden, int heads, int head_dim, int nope, int rope,
                               int latent, float act_eps, const float* mixer_in, float* y, int h, int pos,
                               const AttnSmem& sm) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // 1. current latent -> int8 codes (natural order) and scale, exactly as the up-projection input
  for (int j = tid; j < latent; j += kThreads) sm.xv[j] = ldcg_f(mixer_in + hidden + j);
  __syncthreads();
  const float a_cur = quantize_block(sm.xv, latent, nullptr, 0.0f, 0.0f, act_eps, sm.ql, false, nullptr, sm.red);
  if (h == 0) {
    for (int j = tid; j < latent; j += kThreads) L.latent_q[static_cast<size_t>(pos) * latent + j] = sm.ql[j];
    if (tid == 0) L.latent_scale[pos] = a_cur;
  }
  // 2. RoPE on the query rope part and on k_rope; write k_rope to the cache
  const float sc = L.attn_scale;
  const float* rtab = L.rope + static_cast<size_t>(pos) * rope;  // [rope/2][2]
  for (int jr = tid; jr < rope / 2; jr += kThreads) {
    const float cs = __ldg(rtab + 2 * jr), sn = __ldg(rtab + 2 * jr + 1);
    const float q0 = ldcg_f(mixer_in + h * head_dim + nope + 2 * jr);
    const float q1 = ldcg_f(mixer_in + h * head_dim + nope + 2 * jr + 1);
    const float k0 = ldcg_f(mixer_in + hidden + latent + h * rope + 2 * jr);
    const float k1 = ldcg_f(mixer_in + hidden + latent + h * rope + 2 * jr + 1);
    sm.qr[2 * jr] = (q0 * cs - q1 * sn) * sc;
    sm.qr[2 * jr + 1] = (q0 * sn + q1 * cs) * sc;
    const float kr0 = k0 * cs - k1 * sn, kr1 = k0 * sn + k1 * cs;
    sm.kr[2 * jr] = kr0;
    sm.kr[2 * jr + 1] = kr1;
    uint16_t* kc = L.k_rope_cache + (static_cast<size_t>(pos) * heads + h) * rope;
    kc[2 * jr] = f2h(kr0);
    kc[2 * jr + 1] = f2h(kr1);
  }
  // 3. absorbed query qa[j] = sum_e s*q_nope[e] * W_knope[h*nope+e][j]
  for (int e = tid; e < nope; e += kThreads) sm.qn[e] = ldcg_f(mixer_in + h * head_dim + e) * sc;
  __syncthreads();
  const IvbTernary& kn = L.k_nope_up;
  for (int j = tid; j < latent; j += kThreads) {
    float acc = 0.0f;
    for (int e = 0; e < nope; ++e) {
      const int r = h * nope + e;
      const uint8_t* row = kn.packed + static_cast<size_t>(r) * kn.row_bytes;
      const float w = ternary_code_value(row, j) * h2f(__ldg(kn.scales + static_cast<size_t>(r) * kn.scale_stride + (j >> 7)));
      acc = fmaf(sm.qn[e], w, acc);
    }
    sm.qa[j] = acc;
  }
  float qb = 0.0f;
  if (kn.bias != nullptr) {
    float p = 0.0f;
    for (int e = tid; e < nope; e += kThreads) p = fmaf(sm.qn[e], __ldg(kn.bias + h * nope + e), p);
    qb = block_sum(p, sm.red);
  } else {
    __syncthreads();
  }
  // 4. online softmax over t = warp, warp + 8, ...; lane owns latent j = lane + 32 i
  const int per_lane = (latent + 31) >> 5;
  float u[kMaxLatentPerLane];
#pragma unroll
  for (int i = 0; i < kMaxLatentPerLane; ++i) u[i] = 0.0f;
  float m = -INFINITY, l = 0.0f;
  for (int t = warp; t <= pos; t += kWarps) {
    const bool cur = t == pos;
    const int8_t* qlt = cur ? sm.ql : L.latent_q + static_cast<size_t>(t) * latent;
    const float at = cur ? a_cur : ldcg_f(L.latent_scale + t);
    float codes[kMaxLatentPerLane];
    float part = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxLatentPerLane; ++i) {
      const int j = lane + (i << 5);
      float cval = 0.0f;
      if (i < per_lane && j < latent) cval = static_cast<float>(cur ? qlt[j] : __ldcg(qlt + j));
      codes[i] = cval;
      if (i < per_lane && j < latent) part = fmaf(sm.qa[j], cval, part);
    }
    float rp = 0.0f;
    const uint16_t* krt = L.k_rope_cache + (static_cast<size_t>(t) * heads + h) * rope;
    for (int r = lane; r < rope; r += 32) {
      const float kv = cur ? sm.kr[r] : h2f(__ldcg(krt + r));
      rp = fmaf(sm.qr[r], kv, rp);
    }
    part = warp_sum(part);
    rp = warp_sum(rp);
    const float s = at * part + qb + rp;
    const float mn = fmaxf(m, s);
    const float corr = expf(m - mn);
    const float wgt = expf(s - mn);
    l = l * corr + wgt;
    const float wa = wgt * at;
#pragma unroll
    for (int i = 0; i < kMaxLatentPerLane; ++i) u[i] = u[i] * corr + wa * codes[i];
    m = mn;
  }
  // 5. merge the warps
  float* mine = sm.part + warp * (latent + 2);
#pragma unroll
  for (int i = 0; i < kMaxLatentPerLane; ++i) {
    const int j = lane + (i << 5);
    if (i < per_lane && j < latent) mine[j] = u[i];
  }
  if (lane == 0) {
    mine[latent] = m;
    mine[latent + 1] = l;
  }
  __syncthreads();
  float mm = -INFINITY;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) mm = fmaxf(mm, sm.part[w * (latent + 2) + latent]);
  float ltot = 0.0f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const float mw = sm.part[w * (latent + 2) + latent];
    const float f = mw == -INFINITY ? 0.0f : expf(mw - mm);
    ltot += f * sm.part[w * (latent + 2) + latent + 1];
  }
  for (int j = tid; j < latent; j += kThreads) {
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float mw = sm.part[w * (latent + 2) + latent];
      const float f = mw == -INFINITY ? 0.0f : expf(mw - mm);
      v = fmaf(f, sm.part[w * (latent + 2) + j], v);
    }
    sm.xv[j] = v;  // reuse as the weighted latent sum
  }
  __syncthreads();
  // 6. out_h[e] = W_v[h*hd+e] . u / l + b_v
  const IvbTernary& vu = L.v_up;
  int tpr = kThreads / head_dim;
  if (tpr > 32) tpr = 32;
  int tpr_log = 0;
  while ((2 << tpr_log) <= tpr) ++tpr_log;
  tpr = 1 << tpr_log;
  const float inv_l = 1.0f / ltot;
  for (int base = 0; base < head_dim; base += kThreads >> tpr_log) {
    const int e = base + (tid >> tpr_log);
    const int part_id = tid & (tpr - 1);
    float acc = 0.0f;
    if (e < head_dim) {
      const int r = h * head_dim + e;
      const uint8_t* row = vu.packed + static_cast<size_t>(r) * vu.row_bytes;
      const uint16_t* srow = vu.scales + static_cast<size_t>(r) * vu.scale_stride;
      const int span = (latent + tpr - 1) / tpr;
      const int j0 = part_id * span, j1 = min(latent, j0 + span);
      for (int j = j0; j < j1; ++j) acc = fmaf(ternary_code_value(row, j) * h2f(__ldg(srow + (j >> 7))), sm.xv[j], acc);
    }
    for (int off = 1; off < tpr; off <<= 1) acc += __shfl_xor_sync(kFull, acc, off);
    if (e < head_dim && part_id == 0) {
      float o = acc * inv_l;
      if (vu.bias != nullptr) o += __ldg(vu.bias + h * head_dim + e);
      y[h * head_dim + e] = o;
    }
  }
  __syncthreads();
}

// ------------------------------------------------------------------------------------------------
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy as 1, 2, 3", SC'11).
// ------------------------------------------------------------------------------------------------
__host__ __device__ __forceinline__ float philox_uniform(uint64_t key, uint64_t counter) {
  uint32_t c0 = static_cast<uint32_t>(counter), c1 = static_cast<uint32_t>(counter >> 32);
  uint32_t c2 = 0x49766f6eu, c3 = 0u;
  uint32_t k0 = static_cast<uint32_t>(key), k1 = static_cast<uint32_t>(key >> 32);
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = static_cast<uint64_t>(0xD2511F53u) * c0;
    const uint64_t p1 = static_cast<uint64_t>(0xCD9E8D57u) * c2;
    const uint32_t hi0 = static_cast<uint32_t>(p0 >> 32), lo0 = static_cast<uint32_t>(p0);
    const uint32_t hi1 = static_cast<uint32_t>(p1 >> 32), lo1 = static_cast<uint32_t>(p1);
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return static_cast<float>(c0 >> 8) * (1.0f / 16777216.0f);
}

// ------------------------------------------------------------------------------------------------
// Sampler (one CTA). score = logit * (1/T); seen: score *= score > 0 ? 1/rp : rp.
// Exact top-k by an 8-bit radix select on order-preserving keys (ties: lower index first),
// candidates ordered by (score desc, index asc), p_j = exp(s_j - s_0), canonical CDF (warp
// Hillis-Steele scans over 32-candidate chunks, chunk carries added in order), draw
// target = u * total, token = first j with cdf_j > target.
// Reference: ternary.cu:984-1337, decoder.py:324-333 (_sample), cpu_decoder.py:234-285.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ unsigned order_key(float v) {
  const unsigned b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_value(unsigned k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

struct SampleSmem {
  unsigned* keys;    // [vocab]
  unsigned* hist;    // [kWarps][256]
  unsigned* ckey;    // [kMaxTopK]
  int* cidx;         // [kMaxTopK]
  float* cprob;      // [kMaxTopK]
  int* misc;         // [16]
  float* red;        // [64]
};

static __device__ void sample_block(const float* logits, uint8_t* seen, int vocab, const float* sampling, const int64_t* top_k_ptr,
                             int max_top_k, uint64_t* rng, int64_t* token, int64_t* history, const SampleSmem& sm) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float inv_t = 1.0f / __ldcg(sampling);
  const float pen = __ldcg(sampling + 1), ipen = __ldcg(sampling + 2);
  long long kreq = ldcg_i64(top_k_ptr);
  int cap = min(min(max_top_k, vocab), kMaxTopK);
  const int K = static_cast<int>(kreq < 1 ? 1 : (kreq > cap ? cap : kreq));
  for (int i = tid; i < vocab; i += kThreads) {
    float s = ldcg_f(logits + i) * inv_t;
    if (__ldcg(seen + i)) s *= s > 0.0f ? ipen : pen;
    sm.keys[i] = order_key(s);
  }
  __syncthreads();
  // radix select of the K-th largest key
  unsigned prefix = 0u, mask = 0u;
  int remaining = K;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = tid; b < kWarps * 256; b += kThreads) sm.hist[b] = 0u;
    __syncthreads();
    unsigned* wh = sm.hist + warp * 256;
    for (int base = 0; base < vocab; base += kThreads) {
      const int i = base + tid;
      const bool in = i < vocab && (sm.keys[i] & mask) == prefix;
      const unsigned digit = in ? (sm.keys[i] >> shift) & 255u : 256u;
      const unsigned active = __ballot_sync(kFull, in);
      if (in) {
        const unsigned peers = __match_any_sync(active, digit);
        if (lane == __ffs(peers) - 1) atomicAdd(wh + digit, static_cast<unsigned>(__popc(peers)));
      }
    }
    __syncthreads();
    // thread t owns digit d = 255 - t (descending order) so an inclusive scan counts digits >= d
    const int d = 255 - tid;
    unsigned cnt = 0;
    if (tid < 256) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) cnt += sm.hist[w * 256 + d];
    }
    unsigned incl = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const unsigned o = __shfl_up_sync(kFull, incl, off);
      if (lane >= off) incl += o;
    }
    if (lane == 31) sm.misc[warp] = static_cast<int>(incl);
    __syncthreads();
    unsigned carry = 0;
    for (int w = 0; w < warp; ++w) carry += static_cast<unsigned>(sm.misc[w]);
    incl += carry;
    const unsigned above = incl - cnt;  // keys with a larger digit
    __syncthreads();
    if (tid < 256 && cnt > 0 && static_cast<int>(above) < remaining && remaining <= static_cast<int>(above + cnt)) {
      sm.misc[8] = d;
      sm.misc[9] = remaining - static_cast<int>(above);
    }
    __syncthreads();
    prefix |= static_cast<unsigned>(sm.misc[8]) << shift;
    mask |= 255u << shift;
    remaining = sm.misc[9];
    __syncthreads();
  }
  const unsigned thr = prefix;  // K-th largest key; `remaining` copies of it are taken, lowest index first
  if (tid == 0) {
    sm.misc[10] = 0;  // count of keys > thr
    sm.misc[11] = 0;  // count of keys == thr gathered
  }
  __syncthreads();
  for (int i = tid; i < vocab; i += kThreads) {
    const unsigned k = sm.keys[i];
    if (k > thr) {
      const int slot = atomicAdd(&sm.misc[10], 1);
      sm.ckey[slot] = k;
      sm.cidx[slot] = i;
    }
  }
  __syncthreads();
  const int greater = sm.misc[10];
  if (warp == 0) {
    // ties at the threshold: take the `remaining` lowest indices, scanning in index order
    int taken = 0;
    for (int base = 0; base < vocab && taken < remaining; base += 32) {
      const int i = base + lane;
      const bool eq = i < vocab && sm.keys[i] == thr;
      const unsigned bal = __ballot_sync(kFull, eq);
      const int rank = __popc(bal & ((1u << lane) - 1u));
      if (eq && taken + rank < remaining) {
        sm.ckey[greater + taken + rank] = thr;
        sm.cidx[greater + taken + rank] = i;
      }
      taken += __popc(bal);
    }
  }
  __syncthreads();
  // order candidates by (key desc, index asc): rank by counting
  for (int c = tid; c < K; c += kThreads) {
    const unsigned kc = sm.ckey[c];
    const int ic = sm.cidx[c];
    int rank = 0;
    for (int o = 0; o < K; ++o) {
      const unsigned ko = sm.ckey[o];
      rank += (ko > kc || (ko == kc && sm.cidx[o] < ic)) ? 1 : 0;
    }
    sm.hist[rank] = kc;                        // sorted keys (hist reused, K <= 1024 < 2048)
    sm.hist[kMaxTopK + rank] = static_cast<unsigned>(ic);
  }
  __syncthreads();
  const float top = key_value(sm.hist[0]);
  for (int c = tid; c < K; c += kThreads) sm.cprob[c] = expf(key_value(sm.hist[c]) - top);
  __syncthreads();
  // canonical CDF: per 32-chunk Hillis-Steele inclusive scan, chunk carries added sequentially
  if (warp == 0) {
    float carry = 0.0f;
    for (int base = 0; base < K; base += 32) {
      const int c = base + lane;
      float v = c < K ? sm.cprob[c] : 0.0f;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float o = __shfl_up_sync(kFull, v, off);
        if (lane >= off) v += o;
      }
      if (c < K) sm.cprob[c] = carry + v;
      carry = carry + __shfl_sync(kFull, v, 31);
    }
  }
  __syncthreads();
  const uint64_t key = rng[0], ctr = rng[1];
  const float uval = fminf(philox_uniform(key, ctr), 0.99999994f);
  const float target = uval * sm.cprob[K - 1];
  float below = 0.0f;  // number of candidates whose cdf <= target (cdf is non-decreasing)
  for (int c = tid; c < K; c += kThreads) below += sm.cprob[c] <= target ? 1.0f : 0.0f;
  const int chosen = min(static_cast<int>(block_sum(below, sm.red)), K - 1);
  if (tid == 0) {
    rng[1] = ctr + 1;
    const int index = static_cast<int>(sm.hist[kMaxTopK + chosen]);
    *token = index;
    if (history != nullptr) *history = index;
    seen[index] = 1;
  }
  __syncthreads();
}

// ------------------------------------------------------------------------------------------------
// Bounded grid barrier. Arrival: fence + atomic add on a monotonically growing counter; the CTA
// waits until the counter reaches `target`. The wait gives up after timeout_ns (globaltimer) or when
// another CTA has posted an error, recording IVB_ETIMEOUT in the error word. Returns false on error.
// ------------------------------------------------------------------------------------------------
struct Sync {
  unsigned* counter;
  unsigned* error;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ bool wait_counter(const Sync& s, unsigned target) {
  unsigned long long t0 = 0ull;
  unsigned spins = 0u;
  while (true) {
    const unsigned v = ld_acquire_u32(s.counter);
    if (static_cast<int>(v - target) >= 0) return true;
    ++spins;
    if ((spins & 63u) == 0u && ld_relaxed_u32(s.error) != 0u) return false;
    if ((spins & 255u) == 0u) {
      const unsigned long long t = global_ns();
      if (t0 == 0ull) {
        t0 = t;
      } else if (t - t0 > s.timeout_ns) {
        atomicCAS(s.error, 0u, static_cast<unsigned>(IVB_ETIMEOUT));
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool grid_barrier(const Sync& s, unsigned target, int* flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(s.counter, 1u);
    const bool ok = wait_counter(s, target);
    __threadfence();
    *flag = ok ? 0 : 1;
  }
  __syncthreads();
  return *flag == 0;
}

}  // namespace ivb
