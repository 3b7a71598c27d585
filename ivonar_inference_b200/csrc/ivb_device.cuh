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
// The quantiser's sum of squares keeps a fixed 256-lane order (lane t sums inputs t, t+256, ... with
// fmaf, then a warp butterfly and the warps in order), independent of the CTA size.
constexpr int kCanonLanes = 256;
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

// n floats from global (L2) into shared memory, eight independent loads in flight per thread.
__device__ __forceinline__ void load_vector(const float* __restrict__ src, int n, float* dst) {
  const int tid = threadIdx.x;
  for (int base = 0; base < n; base += 8 * kThreads) {
    float r[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = base + tid + k * kThreads;
      r[k] = i < n ? __ldcg(src + i) : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = base + tid + k * kThreads;
      if (i < n) dst[i] = r[k];
    }
  }
}

// ---- bulk async copies (cp.async.bulk, TMA engine) into shared memory, completed on an mbarrier ----
__device__ __forceinline__ unsigned smem_addr(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
// dst, src 16-byte aligned; bytes a multiple of 16
__device__ __forceinline__ void bulk_copy(void* dst, const void* src, unsigned bytes, unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
// First statement of a kernel launched with launch_pdl: wait until the previous grid on the stream has
// completed and its writes are visible, then let the next grid be scheduled (it waits the same way).
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Timeline mark for tuning: thread 0 stores the globaltimer into marks[slot] when tracing.
__device__ __forceinline__ void mark(unsigned long long* marks, int slot) {
  if (marks != nullptr && threadIdx.x == 0) marks[slot] = global_ns();
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
// Block maximum of non-negative floats: their bit patterns order like the values, so each warp
// reduces with one redux instruction and the warps meet in a shared word (exact; order-free).
__device__ __forceinline__ float block_max_nonneg(float v, float* red) {
  const unsigned m = __reduce_max_sync(kFull, __float_as_uint(v));
  unsigned* slot = reinterpret_cast<unsigned*>(red) + 32;
  if (threadIdx.x == 0) *slot = 0u;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) atomicMax(slot, m);
  __syncthreads();
  const float t = __uint_as_float(*slot);
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

// int32 sum over 64 inputs of code * q8 (codes 0..2 = ternary value + 1). Four independent dp4a
// chains (one per weight word) keep the dependency depth at four.
__device__ __forceinline__ int word_dot(unsigned w, const int4 a) {
  int d = __dp4a(static_cast<int>(w & 0x03030303u), a.x, 0);
  d = __dp4a(static_cast<int>((w >> 2) & 0x03030303u), a.y, d);
  d = __dp4a(static_cast<int>((w >> 4) & 0x03030303u), a.z, d);
  return __dp4a(static_cast<int>((w >> 6) & 0x03030303u), a.w, d);
}
__device__ __forceinline__ int chunk_dot(const uint4 w, const int8_t* act, int u) {
  const int rot = (u >> 1) & 3;
  const char* base = reinterpret_cast<const char*>(act) + (u << 6);
  const int4 a0 = *reinterpret_cast<const int4*>(base + (((0 + rot) & 3) << 4));
  const int4 a1 = *reinterpret_cast<const int4*>(base + (((1 + rot) & 3) << 4));
  const int4 a2 = *reinterpret_cast<const int4*>(base + (((2 + rot) & 3) << 4));
  const int4 a3 = *reinterpret_cast<const int4*>(base + (((3 + rot) & 3) << 4));
  return (word_dot(w.x, a0) + word_dot(w.y, a1)) + (word_dot(w.z, a2) + word_dot(w.w, a3));
}

// rintf(v / scale) without a division per element: y = v * (1 / scale) differs from the true quotient
// v / scale by at most |v / scale| * 2^-23 (two roundings), and the correctly rounded quotient by at
// most half an ulp more. When y is farther than that from every half-integer, both round to the same
// integer; the rare values closer to a half-integer take the IEEE division. |v / scale| <= 128 here.
// quant_code_fast returns the code and sets `near` instead of branching, so a caller can keep its
// loop free of control flow and redo the flagged values afterwards.
__device__ __forceinline__ int quant_code_fast(float v, float rscale, bool& near) {
  const float y = v * rscale;
  const float r = rintf(y);
  near = !(fabsf(fabsf(y - r) - 0.5f) > 4.0e-5f);
  return static_cast<int>(r);
}
__device__ __forceinline__ int quant_code(float v, float scale, float rscale) {
  bool near;
  const int q = quant_code_fast(v, rscale, near);
  return near ? static_cast<int>(rintf(v / scale)) : q;
}

// The 16 two-bit codes of a packed word (input 4b + f in bits 8b + 2f) as exact floats code - 1.
__device__ __forceinline__ void word_codes_m1(unsigned w, float* cm1) {
#pragma unroll
  for (int f = 0; f < 4; ++f) {
    const unsigned m = (w >> (2 * f)) & 0x03030303u;
#pragma unroll
    for (int b = 0; b < 4; ++b)
      cm1[4 * b + f] = __uint_as_float(__byte_perm(m, 0x4B000000u, 0x7440 | b)) - 8388609.0f;
  }
}

// A two-bit ternary code c (0, 1, 2) as the exact float c - 1 without the conversion unit: c placed in
// the low mantissa bits of 2^23, then 2^23 + 1 subtracted.
__device__ __forceinline__ float code_m1(unsigned c) { return __uint_as_float(0x4B000000u | (c & 3u)) - 8388609.0f; }

// Four signed bytes to exact floats without the conversion unit: biased byte b + 128 placed in the
// low mantissa bits of 2^23, then 2^23 + 128 subtracted (exact for every byte value).
__device__ __forceinline__ void bytes_to_f32(unsigned w, float* f) {
  const unsigned b = w ^ 0x80808080u;
  f[0] = __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7440)) - 8388736.0f;
  f[1] = __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7441)) - 8388736.0f;
  f[2] = __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7442)) - 8388736.0f;
  f[3] = __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7443)) - 8388736.0f;
}

// ------------------------------------------------------------------------------------------------
// Canonical per-token int8 quantiser (optionally with RMSNorm: clamp(x * inv_rms, +-clip) * w).
// src holds the fp32 input (n values, shared). For the sum of squares lane t < 256 owns inputs
// t, t+256, ... and accumulates them with fmaf in that order, then block_sum. inv_rms = 1 / sqrtf(ss / n + eps) (IEEE sqrt and divide),
// scale = max(amax / 127, act_eps), code = rintf(v / scale). Writes codes either in the transposed
// GEMV layout (transposed = true) or in natural order, and 64-input chunk sums to xsum (if given).
// Returns the activation scale. Reference: ternary.cu:148-197, cpu_decoder.py:30-70.
// ------------------------------------------------------------------------------------------------
// One compact code path for every n (the decode kernel runs it between many other ops, so its
// instruction footprint matters more than re-reading src): the normalised value is recomputed
// bit-identically in each pass. src is only read (it may be a push target of a later op).
static __device__ float quantize_block(const float* src, int n, const float* norm_w, float norm_eps, float clip,
                                       float act_eps, int8_t* codes, bool transposed, int* xsum, float* red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int chunks = (n + 63) >> 6, padded = chunks << 6;
  // red[0, kWarps): warp partial sums of squares; red[16, 16 + kWarps): warp maxima. Each slot range is
  // written before one barrier and read after it by every thread, and the next write to either range
  // comes after a later barrier of this function, so one barrier per reduction suffices.
  float inv = 0.0f;
  if (norm_w != nullptr) {
    float p = 0.0f;
    if (tid < kCanonLanes) {
#pragma unroll 4
      for (int i = tid; i < n; i += kCanonLanes) {
        const float x = src[i];
        p = fmaf(x, x, p);
      }
    }
    p = warp_sum(p);  // warps beyond the canonical lanes add exact zeros
    if (lane == 0) red[warp] = p;
    __syncthreads();
    float ss = red[0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) ss += red[w];
    inv = 1.0f / sqrtf(ss / static_cast<float>(n) + norm_eps);
  }
  auto value = [&](int i) -> float {
    const float x = src[i];
    return norm_w != nullptr ? __fmul_rn(fminf(fmaxf(__fmul_rn(x, inv), -clip), clip), norm_w[i]) : x;
  };
  float am = 0.0f;
#pragma unroll 4
  for (int i = tid; i < n; i += kThreads) am = fmaxf(am, fabsf(value(i)));
  if (xsum != nullptr)
    for (int u = tid; u < chunks; u += kThreads) xsum[u] = 0;
  // non-negative floats order like their bit patterns: one redux per warp, the warps meet in shared slots
  unsigned* wmax = reinterpret_cast<unsigned*>(red) + 16;
  {
    const unsigned m = __reduce_max_sync(kFull, __float_as_uint(am));
    if (lane == 0) wmax[warp] = m;
  }
  __syncthreads();
  unsigned mbits = wmax[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) mbits = max(mbits, wmax[w]);
  const float amax = __uint_as_float(mbits);
  const float scale = fmaxf(amax / 127.0f, act_eps);
  const float rscale = 1.0f / scale;
  // codes; each warp's 32 consecutive inputs of one pass share a 64-input chunk, so the chunk sums are
  // warp reductions added with shared atomics (integers: the order does not matter)
  bool near = false;
#pragma unroll 4
  for (int base = 0; base < padded; base += kThreads) {
    const int i = base + tid;
    bool nr = false;
    const int q = i < n ? quant_code_fast(value(i), rscale, nr) : 0;
    near |= nr;
    if (i < padded) codes[transposed ? act_slot(i) : i] = static_cast<int8_t>(q);
    if (xsum != nullptr) {
      const int t = __reduce_add_sync(kFull, q);
      if (lane == 0 && i < padded) atomicAdd(xsum + (i >> 6), t);
    }
  }
  if (__syncthreads_or(near)) {
    // rare: values within rounding distance of a half-integer take the IEEE division
    for (int i = tid; i < n; i += kThreads) {
      const float v = value(i);
      bool nr = false;
      const int q = quant_code_fast(v, rscale, nr);
      if (nr) {
        const int qe = static_cast<int>(rintf(v / scale));
        if (qe != q) {
          codes[transposed ? act_slot(i) : i] = static_cast<int8_t>(qe);
          if (xsum != nullptr) atomicAdd(xsum + (i >> 6), qe - q);
        }
      }
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
// pre: residual values of rows [r0, r1) loaded ahead (shared memory) or nullptr.
static __device__ void gemv_rows(const IvbTernary& m, const GemvGeom& g, const int8_t* act, const int* xsum, float act_scale,
                          int epilogue, float* out, uint4 (&pf)[kPrefetch], float (&pfs)[kPrefetch], float* res,
                          const float* pre) {
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
            if (epilogue == IVB_EPI_RESIDUAL) out[r] = (pre != nullptr ? pre[r - g.r0] : ldcg_f(out + r)) + result;
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
// Exactly the reference's softmax(q.k) v with k_nope = up(latent), v = up(latent) (both linear in the
// int8 latent codes); reference ternary.cu:509-611, decoder.py:271-297, attention.py:136-151.
// mixer_in = [q (hidden) | latent (L) | k_rope (heads * rope)].
// Cache layout (device): latent codes [max_len][lpad] int8 (lpad = L rounded up to 16), scales
// [max_len rounded up to 4] fp32, k_rope [heads][max_len][rpad] fp16 (rpad = rope rounded up to 8).
// The head's weight rows and a tile of cached positions are bulk-copied (TMA engine) into shared
// memory; the copies of the first tile are issued before the CTA waits for the entry projection.
// ------------------------------------------------------------------------------------------------
struct AttnGeom {
  int latent, lpad, rope, rpad, nope, head_dim, heads, max_len, tile;
  int kn_rb, kn_ss, v_rb, v_ss;  // row bytes and scale strides of W_knope and W_v
  // byte offsets into the attention shared-memory region
  int o_wkn, o_skn, o_wv, o_sv, o_lat, o_lsc, o_kr, o_qa, o_qr, o_krc, o_qn, o_xv, o_ql, o_sc, o_part, o_red, total;
};

__host__ __device__ inline int round16(int v) { return (v + 15) / 16 * 16; }

__host__ __device__ inline AttnGeom attn_geom(int latent, int rope, int nope, int head_dim, int heads, int max_len,
                                              int kn_rb, int kn_ss, int v_rb, int v_ss, int tile) {
  AttnGeom g;
  g.latent = latent;
  g.lpad = round16(latent);
  g.rope = rope;
  g.rpad = (rope + 7) / 8 * 8;
  g.nope = nope;
  g.head_dim = head_dim;
  g.heads = heads;
  g.max_len = max_len;
  g.tile = tile;
  g.kn_rb = kn_rb;
  g.kn_ss = kn_ss;
  g.v_rb = v_rb;
  g.v_ss = v_ss;
  int o = 0;
  g.o_wkn = o;  o += round16(nope * kn_rb);
  g.o_skn = o;  o += round16(nope * kn_ss * 2);
  g.o_wv = o;   o += round16(head_dim * v_rb);
  g.o_sv = o;   o += round16(head_dim * v_ss * 2);
  g.o_lat = o;  o += round16(tile * g.lpad);
  g.o_lsc = o;  o += round16(((tile + 3) / 4 * 4) * 4);
  g.o_kr = o;   o += round16(tile * g.rpad * 2);
  g.o_qa = o;   o += round16(latent * 4);
  g.o_qr = o;   o += round16(rope * 4);
  g.o_krc = o;  o += round16(rope * 4);
  g.o_qn = o;   o += round16(nope * 4);
  g.o_xv = o;   o += round16(((latent + 63) / 64 * 64) * 4);
  g.o_ql = o;   o += round16((latent + 63) / 64 * 64);
  g.o_sc = o;   o += round16((tile + 1) * 4);
  g.o_part = o; o += round16(kWarps * latent * 4);
  g.o_red = o;  o += round16(64 * 4);
  g.total = o;
  return g;
}

// Thread 0 only: queue the bulk copies of the head's weights (if `weights`) and of cached positions
// [start, start + count) on `bar`.
__device__ __forceinline__ void attn_issue(const IvbLayerDesc& L, const AttnGeom& g, unsigned char* sm, int h, int start,
                                           int count, bool weights, unsigned long long* bar) {
  const unsigned wkn = g.nope * g.kn_rb, skn = g.nope * g.kn_ss * 2, wv = g.head_dim * g.v_rb, sv = g.head_dim * g.v_ss * 2;
  const unsigned lat = count * g.lpad, lsc = ((count + 3) / 4 * 4) * 4, kr = count * g.rpad * 2;
  unsigned bytes = (weights ? wkn + skn + wv + sv : 0u) + (count > 0 ? lat + lsc + kr : 0u);
  asm volatile("fence.proxy.async.global;" ::: "memory");
  fence_proxy_async();
  mbar_expect_tx(bar, bytes);
  if (weights) {
    bulk_copy(sm + g.o_wkn, L.k_nope_up.packed + static_cast<size_t>(h) * g.nope * g.kn_rb, wkn, bar);
    bulk_copy(sm + g.o_skn, L.k_nope_up.scales + static_cast<size_t>(h) * g.nope * g.kn_ss, skn, bar);
    bulk_copy(sm + g.o_wv, L.v_up.packed + static_cast<size_t>(h) * g.head_dim * g.v_rb, wv, bar);
    bulk_copy(sm + g.o_sv, L.v_up.scales + static_cast<size_t>(h) * g.head_dim * g.v_ss, sv, bar);
  }
  if (count > 0) {
    bulk_copy(sm + g.o_lat, L.latent_q + static_cast<size_t>(start) * g.lpad, lat, bar);
    bulk_copy(sm + g.o_lsc, L.latent_scale + start, lsc, bar);
    bulk_copy(sm + g.o_kr, L.k_rope_cache + (static_cast<size_t>(h) * g.max_len + start) * g.rpad, kr, bar);
  }
}

// Bounded wait for the bulk copies on `bar` (phase parity `parity`); false after timeout_ns.
__device__ __forceinline__ bool attn_wait(unsigned long long* bar, unsigned parity, unsigned long long timeout_ns,
                                          unsigned* error) {
  unsigned long long t0 = 0ull;
  unsigned spins = 0u;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 255u) == 0u) {
      const unsigned long long t = global_ns();
      if (t0 == 0ull) {
        t0 = t;
      } else if (t - t0 > timeout_ns) {
        atomicCAS(error, 0u, static_cast<unsigned>(IVB_ETIMEOUT));
        return false;
      }
    }
  }
  return true;
}

__device__ __forceinline__ float code_value(const unsigned char* row, int j) {
  return static_cast<float>(static_cast<int>((row[j >> 2] >> ((j & 3) << 1)) & 3) - 1);
}

// Returns false if a bulk copy did not complete in time. `parity` is the CTA's mbarrier phase bit.
// The caller issued attn_issue(weights = true, tile 0) for this head before the phase started.
static __device__ bool attention_head(const IvbLayerDesc& L, const AttnGeom& g, int hidden, float act_eps,
                                      const float* mixer_in, float* y, int h, int pos, unsigned char* sm,
                                      unsigned long long* bar, unsigned& parity, unsigned long long timeout_ns,
                                      unsigned* error, unsigned long long* marks = nullptr) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int latent = g.latent, rope = g.rope, nope = g.nope, hd = g.head_dim;
  float* qa = reinterpret_cast<float*>(sm + g.o_qa);
  float* qr = reinterpret_cast<float*>(sm + g.o_qr);
  float* krc = reinterpret_cast<float*>(sm + g.o_krc);
  float* qn = reinterpret_cast<float*>(sm + g.o_qn);
  float* xv = reinterpret_cast<float*>(sm + g.o_xv);
  int8_t* qlc = reinterpret_cast<int8_t*>(sm + g.o_ql);
  float* sc = reinterpret_cast<float*>(sm + g.o_sc);
  float* part = reinterpret_cast<float*>(sm + g.o_part);
  float* red = reinterpret_cast<float*>(sm + g.o_red);
  const int8_t* tlat = reinterpret_cast<const int8_t*>(sm + g.o_lat);
  const float* tlsc = reinterpret_cast<const float*>(sm + g.o_lsc);
  const uint16_t* tkr = reinterpret_cast<const uint16_t*>(sm + g.o_kr);
  // 1. current latent -> int8 codes and scale (the up-projection's input quantisation)
  load_vector(mixer_in + hidden, latent, xv);
  __syncthreads();
  const float a_cur = quantize_block(xv, latent, nullptr, 0.0f, 0.0f, act_eps, qlc, false, nullptr, red);
  mark(marks, 1);
  if (h == 0) {
    for (int j = tid; j < latent; j += kThreads) L.latent_q[static_cast<size_t>(pos) * g.lpad + j] = qlc[j];
    if (tid == 0) L.latent_scale[pos] = a_cur;
  }
  // 2. RoPE on the query rope part and on k_rope; append k_rope; scaled query nope part
  const float scl = L.attn_scale;
  const float* rtab = L.rope + static_cast<size_t>(pos) * rope;
  for (int jr = tid; jr < rope / 2; jr += kThreads) {
    const float cs = __ldg(rtab + 2 * jr), sn = __ldg(rtab + 2 * jr + 1);
    const float q0 = __ldcg(mixer_in + h * hd + nope + 2 * jr), q1 = __ldcg(mixer_in + h * hd + nope + 2 * jr + 1);
    const float k0 = __ldcg(mixer_in + hidden + latent + h * rope + 2 * jr);
    const float k1 = __ldcg(mixer_in + hidden + latent + h * rope + 2 * jr + 1);
    qr[2 * jr] = (q0 * cs - q1 * sn) * scl;
    qr[2 * jr + 1] = (q0 * sn + q1 * cs) * scl;
    const float kr0 = k0 * cs - k1 * sn, kr1 = k0 * sn + k1 * cs;
    krc[2 * jr] = kr0;
    krc[2 * jr + 1] = kr1;
    uint16_t* kc = L.k_rope_cache + (static_cast<size_t>(h) * g.max_len + pos) * g.rpad;
    kc[2 * jr] = f2h(kr0);
    kc[2 * jr + 1] = f2h(kr1);
  }
  for (int e = tid; e < nope; e += kThreads) qn[e] = __ldcg(mixer_in + h * hd + e) * scl;
  asm volatile("fence.proxy.async.global;" ::: "memory");
  // 3. weights and the first cache tile
  if (!attn_wait(bar, parity, timeout_ns, error)) return false;
  parity ^= 1u;
  __syncthreads();
  mark(marks, 2);
  // 4. absorbed query qa[j] = sum_e qn[e] * W_knope[e][j]
  const unsigned char* wkn = sm + g.o_wkn;
  const uint16_t* skn = reinterpret_cast<const uint16_t*>(sm + g.o_skn);
  for (int j = tid; j < latent; j += kThreads) {
    float acc = 0.0f;
    for (int e = 0; e < nope; ++e) acc = fmaf(qn[e], code_value(wkn + e * g.kn_rb, j) * h2f(skn[e * g.kn_ss + (j >> 7)]), acc);
    qa[j] = acc;
  }
  float qb = 0.0f;
  if (L.k_nope_up.bias != nullptr) {
    float p = 0.0f;
    for (int e = tid; e < nope; e += kThreads) p = fmaf(qn[e], __ldg(L.k_nope_up.bias + h * nope + e), p);
    qb = block_sum(p, red);
  } else {
    __syncthreads();
  }
  mark(marks, 3);
  // 5. scores / softmax / weighted latent sum over cache tiles (the current position ends the last one)
  const int per_lane = (latent + 31) >> 5;
  float qa_r[kMaxLatentPerLane];
  float u[kMaxLatentPerLane];
#pragma unroll
  for (int i = 0; i < kMaxLatentPerLane; ++i) {
    const int j = lane + (i << 5);
    qa_r[i] = (i < per_lane && j < latent) ? qa[j] : 0.0f;
    u[i] = 0.0f;
  }
  float m_run = -INFINITY, l_run = 0.0f;
  const int n_tiles = pos == 0 ? 1 : (pos + g.tile - 1) / g.tile;
  for (int ti = 0; ti < n_tiles; ++ti) {
    const int start = ti * g.tile;
    const int count = min(g.tile, pos - start);
    const bool last = ti == n_tiles - 1;
    if (ti > 0) {
      if (tid == 0) attn_issue(L, g, sm, h, start, count, false, bar);
      if (!attn_wait(bar, parity, timeout_ns, error)) return false;
      parity ^= 1u;
    }
    const int npos = count + (last ? 1 : 0);
    for (int k = warp; k < npos; k += kWarps) {
      const bool cur = k == count;
      const int8_t* ql = cur ? qlc : tlat + k * g.lpad;
      const float at = cur ? a_cur : tlsc[k];
      float dot = 0.0f;
#pragma unroll
      for (int i = 0; i < kMaxLatentPerLane; ++i) {
        const int j = lane + (i << 5);
        if (i < per_lane && j < latent) dot = fmaf(qa_r[i], static_cast<float>(ql[j]), dot);
      }
      float rp = 0.0f;
      for (int r = lane; r < rope; r += 32) rp = fmaf(qr[r], cur ? krc[r] : h2f(tkr[k * g.rpad + r]), rp);
      dot = warp_sum(dot);
      rp = warp_sum(rp);
      if (lane == 0) sc[k] = at * dot + qb + rp;
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int k = tid; k < npos; k += kThreads) mx = fmaxf(mx, sc[k]);
    mx = block_max(mx, red);
    const float m_new = fmaxf(m_run, mx);
    const float corr = m_run == -INFINITY ? 0.0f : expf(m_run - m_new);
    float ls = 0.0f;
    for (int k = tid; k < npos; k += kThreads) {
      const float e = expf(sc[k] - m_new);
      sc[k] = e;
      ls += e;
    }
    ls = block_sum(ls, red);
    l_run = l_run * corr + ls;
#pragma unroll
    for (int i = 0; i < kMaxLatentPerLane; ++i) u[i] *= corr;
    for (int k = warp; k < npos; k += kWarps) {
      const bool cur = k == count;
      const int8_t* ql = cur ? qlc : tlat + k * g.lpad;
      const float ea = sc[k] * (cur ? a_cur : tlsc[k]);
#pragma unroll
      for (int i = 0; i < kMaxLatentPerLane; ++i) {
        const int j = lane + (i << 5);
        if (i < per_lane && j < latent) u[i] = fmaf(ea, static_cast<float>(ql[j]), u[i]);
      }
    }
    m_run = m_new;
    __syncthreads();
  }
  mark(marks, 4);
  // 6. merge the warps' partial sums (warps in order)
#pragma unroll
  for (int i = 0; i < kMaxLatentPerLane; ++i) {
    const int j = lane + (i << 5);
    if (i < per_lane && j < latent) part[warp * latent + j] = u[i];
  }
  __syncthreads();
  for (int j = tid; j < latent; j += kThreads) {
    float v = part[j];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) v += part[w * latent + j];
    xv[j] = v;
  }
  __syncthreads();
  mark(marks, 5);
  // 7. out_h[e] = W_v[h*hd+e] . u / l + b_v
  const unsigned char* wv = sm + g.o_wv;
  const uint16_t* sv = reinterpret_cast<const uint16_t*>(sm + g.o_sv);
  int tpr = kThreads / hd;
  if (tpr > 32) tpr = 32;
  int tpr_log = 0;
  while ((2 << tpr_log) <= tpr) ++tpr_log;
  tpr = 1 << tpr_log;
  const float inv_l = 1.0f / l_run;
  for (int base = 0; base < hd; base += kThreads >> tpr_log) {
    const int e = base + (tid >> tpr_log);
    const int pid = tid & (tpr - 1);
    float acc = 0.0f;
    if (e < hd) {
      const unsigned char* row = wv + e * g.v_rb;
      const int span = (latent + tpr - 1) / tpr;
      const int j0 = pid * span, j1 = min(latent, j0 + span);
      for (int j = j0; j < j1; ++j) acc = fmaf(code_value(row, j) * h2f(sv[e * g.v_ss + (j >> 7)]), xv[j], acc);
    }
    for (int off = 1; off < tpr; off <<= 1) acc += __shfl_xor_sync(kFull, acc, off);
    if (e < hd && pid == 0) {
      float o = acc * inv_l;
      if (L.v_up.bias != nullptr) o += __ldg(L.v_up.bias + h * hd + e);
      y[h * hd + e] = o;
    }
  }
  __syncthreads();
  return true;
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
// e^x (x <= 0) for the sampler's candidate weights, written the same way in the kernels and in the CPU
// oracle so that both weigh the candidates bit for bit alike (the libraries' expf differ in the last
// bits, which moves draws that land next to a CDF boundary). Cody-Waite reduction x = n ln2 + r with
// ln2 split into a 12-bit head (n * head is exact) and a tail, e^r by its degree-7 Taylor polynomial in
// Horner form with fused multiply-adds (|r| <= ln2 / 2: truncation below 6e-9 relative), then 2^n
// from the exponent field. Inputs below -87 (weights under 2^-125 against the top candidate's 1) give 0.
__device__ __forceinline__ float sample_exp(float x) {
  if (!(x >= -87.0f)) return 0.0f;
  const float n = rintf(__fmul_rn(x, 0x1.715476p+0f));
  const float r = fmaf(-n, 0x1.0bfbe8p-15f, fmaf(-n, 0x1.62ep-1f, x));
  float p = 0x1.a01a02p-13f;
  p = fmaf(p, r, 0x1.6c16c2p-10f);
  p = fmaf(p, r, 0x1.111112p-7f);
  p = fmaf(p, r, 0x1.555556p-5f);
  p = fmaf(p, r, 0x1.555556p-3f);
  p = fmaf(p, r, 0x1p-1f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  return __fmul_rn(p, __int_as_float((static_cast<int>(n) + 127) << 23));
}
__device__ __forceinline__ float key_value(unsigned k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

constexpr int kCompact = 4096;  // candidates kept after the first radix pass when they fit

struct SampleSmem {
  unsigned* keys;    // [vocab]
  unsigned* hist;    // [kWarps][256]
  unsigned* ckey;    // [kMaxTopK]
  int* cidx;         // [kMaxTopK]
  float* cprob;      // [kMaxTopK]
  unsigned* pkey;    // [kCompact] keys sharing the selected prefix
  int* pidx;         // [kCompact]
  int* misc;         // [16]
  float* red;        // [64]
};

__host__ __device__ inline size_t sample_smem_bytes(int vocab) {
  return static_cast<size_t>(vocab) * 4 + kWarps * 256 * 4 + kMaxTopK * 12 + kCompact * 8 + 16 * 4 + 64 * 4 + 16;
}

__device__ __forceinline__ void carve_sample(unsigned char* smem, int vocab, SampleSmem& sm) {
  sm.keys = reinterpret_cast<unsigned*>(smem);
  sm.hist = sm.keys + vocab;
  sm.ckey = sm.hist + kWarps * 256;
  sm.cidx = reinterpret_cast<int*>(sm.ckey + kMaxTopK);
  sm.cprob = reinterpret_cast<float*>(sm.cidx + kMaxTopK);
  sm.pkey = reinterpret_cast<unsigned*>(sm.cprob + kMaxTopK);
  sm.pidx = reinterpret_cast<int*>(sm.pkey + kCompact);
  sm.misc = sm.pidx + kCompact;
  sm.red = reinterpret_cast<float*>(sm.misc + 16);
}

__device__ __forceinline__ unsigned score_key(float logit, unsigned char flag, float inv_t, float pen, float ipen) {
  float s = logit * inv_t;
  if (flag) s *= s > 0.0f ? ipen : pen;
  return order_key(s);
}

// One 8-bit radix digit over `n` keys (from `keys`, or from the compact list when compact): histogram
// of the digit at `shift` among keys matching prefix/mask, then the digit holding the remaining-th
// largest key. Updates prefix, mask, remaining; returns the count of keys in the selected bin.
static __device__ int radix_digit(const SampleSmem& sm, const unsigned* keys, int n, int shift, unsigned& prefix, unsigned& mask,
                           int& remaining) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int b = tid; b < kWarps * 256; b += kThreads) sm.hist[b] = 0u;
  __syncthreads();
  unsigned* wh = sm.hist + warp * 256;
  for (int base = 0; base < n; base += kThreads) {
    const int i = base + tid;
    const unsigned key = i < n ? keys[i] : 0u;
    const bool in = i < n && (key & mask) == prefix;
    const unsigned digit = in ? (key >> shift) & 255u : 256u;
    const unsigned active = __ballot_sync(kFull, in);
    if (in) {
      const unsigned peers = __match_any_sync(active, digit);
      if (lane == __ffs(peers) - 1) atomicAdd(wh + digit, static_cast<unsigned>(__popc(peers)));
    }
  }
  __syncthreads();
  // thread t owns digit d = 255 - t (descending) so an inclusive scan counts keys with digit >= d
  const int d = 255 - tid;
  unsigned cnt = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) cnt += sm.hist[w * 256 + d];
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
  const unsigned above = incl - cnt;
  if (cnt > 0 && static_cast<int>(above) < remaining && remaining <= static_cast<int>(above + cnt)) {
    sm.misc[8] = d;
    sm.misc[9] = remaining - static_cast<int>(above);
    sm.misc[12] = static_cast<int>(cnt);
  }
  __syncthreads();
  prefix |= static_cast<unsigned>(sm.misc[8]) << shift;
  mask |= 255u << shift;
  remaining = sm.misc[9];
  const int bin = sm.misc[12];
  __syncthreads();
  return bin;
}

// The K best of keys[0, n) (sm.keys) by (key desc, index asc): sm.hist[r] gets the key of rank r and
// sm.hist[kMaxTopK + r] its index. Radix select of the K-th largest key (first digit over all keys, the
// rest over a compact list when the selected bin fits), then a gather and a rank-by-counting order.
static __device__ void select_topk(const SampleSmem& sm, int vocab, int K, unsigned long long* marks = nullptr) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // radix select of the K-th largest key: first digit over all keys, the rest over a compact list
  unsigned prefix = 0u, mask = 0u;
  int remaining = K;
  const int bin = radix_digit(sm, sm.keys, vocab, 24, prefix, mask, remaining);
  mark(marks, 2);
  if (bin <= kCompact) {
    if (tid == 0) sm.misc[13] = 0;
    __syncthreads();
    for (int i = tid; i < vocab; i += kThreads) {
      const unsigned k = sm.keys[i];
      if ((k & mask) == prefix) {
        const int slot = atomicAdd(&sm.misc[13], 1);
        sm.pkey[slot] = k;
        sm.pidx[slot] = i;
      }
    }
    __syncthreads();
    for (int shift = 16; shift >= 0; shift -= 8) radix_digit(sm, sm.pkey, bin, shift, prefix, mask, remaining);
  } else {
    for (int shift = 16; shift >= 0; shift -= 8) radix_digit(sm, sm.keys, vocab, shift, prefix, mask, remaining);
  }
  mark(marks, 3);
  const unsigned thr = prefix;  // the K-th largest key; `remaining` copies of it are taken
  if (tid == 0) {
    sm.misc[10] = 0;  // keys > thr gathered
    sm.misc[11] = 0;  // keys == thr counted
  }
  __syncthreads();
  for (int i = tid; i < vocab; i += kThreads) {
    const unsigned k = sm.keys[i];
    if (k > thr) {
      const int slot = atomicAdd(&sm.misc[10], 1);
      sm.ckey[slot] = k;
      sm.cidx[slot] = i;
    } else if (k == thr) {
      atomicAdd(&sm.misc[11], 1);
    }
  }
  __syncthreads();
  const int greater = sm.misc[10];
  const int ties = sm.misc[11];
  if (ties == remaining) {
    // every key equal to the threshold is taken
    if (tid == 0) sm.misc[14] = 0;
    __syncthreads();
    for (int i = tid; i < vocab; i += kThreads) {
      if (sm.keys[i] == thr) {
        const int slot = greater + atomicAdd(&sm.misc[14], 1);
        sm.ckey[slot] = thr;
        sm.cidx[slot] = i;
      }
    }
  } else if (warp == 0) {
    // more ties than places: the lowest indices win, scanned in index order
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
  mark(marks, 4);
  // order candidates by (key desc, index asc): rank by counting
  for (int c = tid; c < K; c += kThreads) {
    const unsigned kc = sm.ckey[c];
    const int ic = sm.cidx[c];
    int rank = 0;
    for (int o = 0; o < K; ++o) {
      const unsigned ko = sm.ckey[o];
      rank += (ko > kc || (ko == kc && sm.cidx[o] < ic)) ? 1 : 0;
    }
    sm.hist[rank] = kc;
    sm.hist[kMaxTopK + rank] = static_cast<unsigned>(ic);
  }
  __syncthreads();
  mark(marks, 5);
}

// The Philox draw over the K candidates that select_topk ordered: probabilities exp(v - top) of their
// scores, the canonical CDF (per 32-chunk inclusive scan, chunk carries added in order) and the count of
// CDF entries at or below u * total. Returns the chosen rank (the same in every thread); thread 0
// advances the draw counter rng[1].
static __device__ int draw_sorted(const SampleSmem& sm, int K, uint64_t* rng, unsigned long long* marks = nullptr) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float top = key_value(sm.hist[0]);
  for (int c = tid; c < K; c += kThreads) sm.cprob[c] = sample_exp(key_value(sm.hist[c]) - top);
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
  mark(marks, 6);
  const uint64_t key = rng[0], ctr = rng[1];
  const float uval = fminf(philox_uniform(key, ctr), 0.99999994f);
  const float target = uval * sm.cprob[K - 1];
  float below = 0.0f;  // number of candidates whose cdf <= target (cdf is non-decreasing)
  for (int c = tid; c < K; c += kThreads) below += sm.cprob[c] <= target ? 1.0f : 0.0f;
  const int chosen = min(static_cast<int>(block_sum(below, sm.red)), K - 1);
  __syncthreads();  // every thread has read the draw counter
  if (tid == 0) rng[1] = ctr + 1;
  return chosen;
}

static __device__ void sample_block(const float* logits, uint8_t* seen, int vocab, const float* sampling, const int64_t* top_k_ptr,
                                    int max_top_k, uint64_t* rng, int64_t* token, int64_t* history, const SampleSmem& sm,
                                    unsigned long long* marks = nullptr) {
  const int tid = threadIdx.x;
  const float inv_t = 1.0f / __ldcg(sampling);
  const float pen = __ldcg(sampling + 1), ipen = __ldcg(sampling + 2);
  const long long kreq = ldcg_i64(top_k_ptr);
  const int cap = min(min(max_top_k, vocab), kMaxTopK);
  const int K = static_cast<int>(kreq < 1 ? 1 : (kreq > cap ? cap : kreq));
  // scores -> order-preserving keys, four logits and flags per load, four loads in flight
  const int n4 = vocab >> 2;
  const float4* l4 = reinterpret_cast<const float4*>(logits);
  const uchar4* f4 = reinterpret_cast<const uchar4*>(seen);
  for (int base = 0; base < n4; base += 4 * kThreads) {
    float4 lv[4];
    uchar4 fv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int q = base + tid + u * kThreads;
      if (q < n4) {
        lv[u] = __ldcg(l4 + q);
        fv[u] = __ldcg(f4 + q);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int q = base + tid + u * kThreads;
      if (q < n4) {
        sm.keys[4 * q] = score_key(lv[u].x, fv[u].x, inv_t, pen, ipen);
        sm.keys[4 * q + 1] = score_key(lv[u].y, fv[u].y, inv_t, pen, ipen);
        sm.keys[4 * q + 2] = score_key(lv[u].z, fv[u].z, inv_t, pen, ipen);
        sm.keys[4 * q + 3] = score_key(lv[u].w, fv[u].w, inv_t, pen, ipen);
      }
    }
  }
  for (int i = 4 * n4 + tid; i < vocab; i += kThreads) sm.keys[i] = score_key(__ldcg(logits + i), __ldcg(seen + i), inv_t, pen, ipen);
  __syncthreads();
  mark(marks, 1);
  select_topk(sm, vocab, K, marks);
  const int chosen = draw_sorted(sm, K, rng, marks);
  if (tid == 0) {
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
    const unsigned v = ld_relaxed_u32(s.counter);
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
