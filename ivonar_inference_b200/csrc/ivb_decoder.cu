// Whole-GPU persistent decode kernel of libivonar_b200.so.
//
// One cooperative launch of G CTAs (one per SM) runs `steps` tokens: for every token the CTAs walk an
// op program built on the host — per block: fused norm+quantise+GEMV entry projection (with the
// recurrent step of the CTA's head for mamba blocks), the latent attention of the CTA's head (mla
// blocks), the out projection with residual add, the SwiGLU gate/up GEMV and the down GEMV with
// residual add — then the LM head and the sampler. Consecutive ops hand their outputs over through
// flag words in global memory (ivb_decode.cuh: the payload and the token epoch in one 8-byte word,
// gathered by polling), and each CTA's weights stream into a shared-memory ring ahead of use, so the
// weight traffic overlaps the handoff latency. This replaces the reference's 131-137 launches per
// token and its 16-token CUDA graph (kernel_decoder.py:179-283, 683-735).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "ivb_common.h"
#include "ivb_decode.cuh"

size_t ivb_sample_smem_bytes(int vocab);
size_t ivb_gemv_smem_bytes(int n);
int ivb_lpr_log(int in_features);

namespace ivb {

__device__ __forceinline__ void cp_async_f32(float* dst, const float* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }


// Bounded wait on an attention tile mbarrier; the verdict is uniform across the CTA.
__device__ __forceinline__ bool tile_wait(unsigned long long* bar, unsigned parity, unsigned long long timeout_ns) {
  const bool late = !mbar_wait_bounded(bar, parity, timeout_ns);
  return !__syncthreads_or(late);
}

// Tile buffer b of the attention op: tile + 1 key rows, then tile + 1 value rows (head_dim padded to
// kvpad floats); the last tile also holds the current position.
struct TileBuf {
  float* k;  // [tile + 1][kvpad]
  float* v;  // [tile + 1][kvpad]
};

__host__ __device__ __forceinline__ size_t tile_bytes(int tile, int kvpad) {
  return (static_cast<size_t>(tile + 1) * kvpad * 4 + 15) / 16 * 16;
}

__device__ __forceinline__ TileBuf tile_buf(unsigned char* base, const DecodeDims& D, int b) {
  const size_t one = tile_bytes(D.tile, D.kvpad);
  TileBuf tb;
  tb.k = reinterpret_cast<float*>(base + 2 * b * one);
  tb.v = reinterpret_cast<float*>(base + (2 * b + 1) * one);
  return tb;
}

// thread 0: bulk-copy the cached keys and values of positions [start, start + count) of head h into
// tile buffer b (rows of kvpad floats, a multiple of 16 bytes at 16-byte aligned addresses), and mark
// the buffer's copy pending. The rows were written by generic stores of earlier tokens (or kernels).
__device__ __forceinline__ void tile_issue(const IvbLayerDesc& L, const DecodeDims& D, const TileBuf& tb, int h, int start,
                                           int count, unsigned long long* bar, unsigned& pending, int b) {
  const unsigned bytes = static_cast<unsigned>(count) * static_cast<unsigned>(D.kvpad) * 4u;
  const size_t row0 = (static_cast<size_t>(h) * D.max_len + start) * D.kvpad;
  asm volatile("fence.proxy.async.global;" ::: "memory");
  fence_proxy_async();
  mbar_expect_tx(bar, 2u * bytes);
  bulk_copy(tb.k, L.k_cache + row0, bytes, bar);
  bulk_copy(tb.v, L.v_cache + row0, bytes, bar);
  pending |= 1u << b;
}

// Candidate slots of the sampler: every CTA of the head op publishes exactly kp (even) candidates,
// padded with key 0 (below every real score key) where it has fewer rows; the head op's buffer holds
// all CTAs' keys first ([R][kp]) and then all their ids, so a merge gathers straight into a key array
// and an id array. Merge leaders publish kq candidates each the same way.
__device__ __forceinline__ int cand_slots(int K, int rows_per) { return (min(K, max(rows_per, 1)) + 1) & ~1; }

// Publish the first k of (keys, ids) into slots [0, kp) of key_dst and id_dst, padding the rest with
// key 0 and distinct ids pad_id + j (beyond any vocabulary index, so a merge's (key, id) order stays
// total). A final merge always holds at least K real candidates, so padding is never drawn.
__device__ __forceinline__ void cand_put(unsigned long long* key_dst, unsigned long long* id_dst, const unsigned* keys,
                                        const int* ids, int k, int kp, unsigned pad_id, unsigned flag) {
  for (int j = threadIdx.x; j < kp; j += kThreads) {
    ll_store(key_dst + j, j < k ? keys[j] : 0u, flag);
    ll_store(id_dst + j, j < k ? static_cast<unsigned>(ids[j]) : pad_id + static_cast<unsigned>(j), flag);
  }
}

// Gather + (RMSNorm +) quantise of an input of at most E * 256 values, all in registers: thread t polls
// the words t, t + 256, t + 512, ... of the input's flag-word buffer, exactly the elements the canonical
// quantiser assigns to lane t, so the sum of squares (fmaf in that order, warp butterfly, warps in
// order), the amax and the codes (rint(v / scale), transposed GEMV layout, zero padding to a 64-input
// chunk) equal quantize_block's bit for bit. buf == nullptr: the values are read from `keep`; otherwise
// they are also stored there. Returns the activation scale, or -1 in every thread when a word did not
// arrive within timeout_ns. E = 4 serves inputs up to 1024 values, E = 12 up to 3072. xhalf[2u + h] gets
// the sum of the codes of half h of 64-input chunk u (the row dots subtract the chunk's sum).
constexpr int kMaxEPT = 12;  // input elements per thread: n <= 3072
template <int E>
__device__ __forceinline__ float gather_quantize_reg(const unsigned long long* buf, int n, unsigned flag, float* keep,
                                                     const float* norm_w, float norm_eps, float clip, float act_eps,
                                                     int8_t* codes, int* xhalf, float* red, unsigned long long timeout_ns,
                                                     long long* t_arrived) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float x[E];
  bool late = false;
  if (buf != nullptr) {
    unsigned long long w[E];
#pragma unroll
    for (int k = 0; k < E; ++k) {
      const int i = tid + k * kThreads;
      w[k] = i < n ? ll_load1(buf + i) : static_cast<unsigned long long>(flag) << 32;
    }
    unsigned long long t0 = 0ull;
    unsigned spins = 0u;
    while (!late) {
      bool miss = false;
#pragma unroll
      for (int k = 0; k < E; ++k) {
        if (static_cast<unsigned>(w[k] >> 32) != flag) {
          miss = true;
          w[k] = ll_load1(buf + tid + k * kThreads);
        }
      }
      if (!miss) break;
      if ((++spins & 63u) == 0u) {
        const unsigned long long t = global_ns();
        if (t0 == 0ull) t0 = t;
        else if (t - t0 > timeout_ns) late = true;
      }
    }
#pragma unroll
    for (int k = 0; k < E; ++k) {
      const int i = tid + k * kThreads;
      x[k] = __uint_as_float(static_cast<unsigned>(w[k]));
      if (keep != nullptr && i < n) keep[i] = x[k];
    }
  } else {
#pragma unroll
    for (int k = 0; k < E; ++k) {
      const int i = tid + k * kThreads;
      x[k] = i < n ? keep[i] : 0.0f;
    }
  }
  float inv = 0.0f;
  if (norm_w != nullptr) {
    float p2 = 0.0f;
#pragma unroll
    for (int k = 0; k < E; ++k)
      if (tid + k * kThreads < n) p2 = fmaf(x[k], x[k], p2);
    p2 = warp_sum(p2);
    if (lane == 0) red[warp] = p2;
  }
  if (__syncthreads_or(late)) return -1.0f;
  if (t_arrived != nullptr && threadIdx.x == 0) *t_arrived = clock64();  // tracing: the whole input is here
  if (norm_w != nullptr) {
    float ss = red[0];
#pragma unroll
    for (int w2 = 1; w2 < kWarps; ++w2) ss += red[w2];
    inv = 1.0f / sqrtf(ss / static_cast<float>(n) + norm_eps);
  }
  float v[E];
  float am = 0.0f;
#pragma unroll
  for (int k = 0; k < E; ++k) {
    const int i = tid + k * kThreads;
    v[k] = 0.0f;
    if (i < n) v[k] = norm_w != nullptr ? __fmul_rn(fminf(fmaxf(__fmul_rn(x[k], inv), -clip), clip), norm_w[i]) : x[k];
    am = fmaxf(am, fabsf(v[k]));
  }
  unsigned* wmax = reinterpret_cast<unsigned*>(red) + 16;
  {
    const unsigned m = __reduce_max_sync(kFull, __float_as_uint(am));
    if (lane == 0) wmax[warp] = m;
  }
  __syncthreads();
  unsigned mbits = wmax[0];
#pragma unroll
  for (int w2 = 1; w2 < kWarps; ++w2) mbits = max(mbits, wmax[w2]);
  const float scale = fmaxf(__uint_as_float(mbits) / 127.0f, act_eps);
  const float rscale = 1.0f / scale;
  const int padded = (n + 63) & ~63;
  // every code first (the rare value within rounding distance of a half takes the IEEE division), so
  // the E warp reductions below run back to back after one reconvergence
  int qk[E];
  bool near = false;
#pragma unroll
  for (int k = 0; k < E; ++k) {
    bool nr = false;
    qk[k] = tid + k * kThreads < n ? quant_code_fast(v[k], rscale, nr) : 0;
    near |= nr;
  }
  if (near) {
#pragma unroll
    for (int k = 0; k < E; ++k) {
      bool nr = false;
      if (tid + k * kThreads < n) {
        quant_code_fast(v[k], rscale, nr);
        if (nr) qk[k] = static_cast<int>(rintf(v[k] / scale));
      }
    }
  }
  // the code sum of the half chunk each warp holds (64-input chunk u = 4k + warp / 2), for the row dots
  int hs[E];
#pragma unroll
  for (int k = 0; k < E; ++k) hs[k] = __reduce_add_sync(kFull, qk[k]);
#pragma unroll
  for (int k = 0; k < E; ++k) {
    const int i = tid + k * kThreads;
    if (i < padded) codes[act_slot(i)] = static_cast<int8_t>(qk[k]);
    if (lane == 0 && k * kThreads + warp * 32 < padded) xhalf[2 * (4 * k + (warp >> 1)) + (warp & 1)] = hs[k];
  }
  __syncthreads();
  return scale;
}

// Per-CTA state of the decode kernel that the op routines share. It lives in shared memory (thread 0
// writes it, barriers publish it), so the routines compiled out of line read it without touching the
// thread stack, whose local-memory traffic would go to L2 (shared memory takes nearly all of L1 here).
struct Ctx {
  const DecodeParams* p;
  Stream* st;
  unsigned chunk_base;  // stream chunks consumed by the tokens before this one
  unsigned rank;
  float *resid, *loc, *red, *xl, *stg, *rope_s, *seen_s;
  int8_t* act;
  int* xsum;
  unsigned char* U;
  unsigned long long* abar;
  unsigned apar[2];     // phase parities of the two attention tile barriers (flipped by thread 0)
  unsigned apend;       // bit b: a copy into tile buffer b was issued and not yet waited for (thread 0)
  int ssm_row0;         // GEMV CTA: (head * state_dim) * head_dim + first channel in the head (recurrent state rows)
  long long pos;
  unsigned flag;
  int K, kp, kq, n_groups;
  bool two_level, sampling;
  float inv_t, pen, ipen;
  // tracing (thread 0): slots 1..6 of the op's record sum SM cycles spent in six parts of the op
  unsigned long long* marks;
  long long prof[6];
  long long prof_t, prof_t2;
  __device__ __forceinline__ void tick(int part) {
    if (threadIdx.x == 0 && marks != nullptr) {
      const long long now = clock64();
      prof[part] += now - prof_t;
      prof_t = now;
    }
  }
  __device__ __forceinline__ void fail(unsigned code) {
    if (threadIdx.x == 0) atomicCAS(p->error, 0u, code);
  }
};

// The kernel is compiled twice: with kTrace the op routines record their per-part cycle counts (the
// per-op device timeline of ivb_decoder_trace); without it they contain no tracing code at all.
template <bool kTrace>
__device__ __forceinline__ void tick(Ctx& c, int part) {
  if constexpr (kTrace) c.tick(part);
}

// Shared-memory layout of the attention op inside the union region (the plan sizes it the same way):
// kv rows of this position [nope + head_dim] | scaled query, rope pairs rotated [kvpad] | this
// position's key row [kvpad] | the warps' value sums [4 * kThreads] | 16-byte aligned double tile
// buffer (tile_buf).
struct AttnSmem {
  float *kv, *q, *kcur, *part;
  unsigned char* tiles;
};
__host__ __device__ __forceinline__ int r4(int n) { return (n + 3) & ~3; }
__host__ __device__ __forceinline__ size_t attn_fixed_bytes(int nope, int hd) {
  const int kvpad = r4(hd);
  return static_cast<size_t>(r4(nope + hd) + 2 * kvpad + 4 * kThreads) * 4 + 16;
}
__device__ __forceinline__ AttnSmem attn_smem(unsigned char* U, const DecodeDims& D) {
  AttnSmem a;
  a.kv = reinterpret_cast<float*>(U);
  a.q = a.kv + r4(D.nope + D.head_dim);
  a.kcur = a.q + D.kvpad;
  a.part = a.kcur + D.kvpad;
  unsigned char* t = reinterpret_cast<unsigned char*>(a.part + 4 * kThreads);
  a.tiles = t + ((16 - (reinterpret_cast<uintptr_t>(t) & 15)) & 15);
  return a;
}

// thread 0, after a failed wait: let the tile copies still in flight land (bounded) before the shared
// memory they write is reused or released.
__device__ __forceinline__ void attn_drain(Ctx& c, unsigned long long timeout_ns) {
  for (int b = 0; b < 2; ++b)
    if (c.apend & (1u << b)) {
      if (mbar_wait_bounded(&c.abar[b], c.apar[b], timeout_ns)) c.apar[b] ^= 1u;
      c.apend &= ~(1u << b);
    }
}

// The tile loop of the attention op: positions 0..P in tiles (the current position as the extra last
// row of the last tile; the caller issued the copies of tiles 0 and 1), each warp running its own
// online softmax over its positions 32 i + 4 w + g of every tile (lane group g = lane / 8), so a tile
// needs no CTA-wide reduction. Scores: 8 lanes per position, lane q taking the key quads q, q + 8, ...
// against the query quads it holds (one 16-byte load phase is one position's 128 contiguous bytes),
// added by a butterfly over the group. Value sum: lane l owns the value pairs l, l + 32, ... of every
// position the warp holds (a warp reads whole rows). Results per warp: the running maximum m_run, the
// total l_run (scaled by exp(-m_run)) and the value pairs acc. Returns false when a tile's wait ran out.
template <int NQ, int NV>
__device__ __forceinline__ bool attn_tiles(Ctx& c, const DecodeParams& p, const DecodeDims& D, const IvbLayerDesc& L,
                                           const AttnSmem& A, int h, int P, float& m_run, float& l_run, float2 (&acc)[NV]) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 3, q = lane & 7;
  const int kq = D.kvpad >> 2, kv2 = D.kvpad >> 1, tile = D.tile, kvpad = D.kvpad, hd = D.head_dim, nope = D.nope;
  unsigned long long* const abar = c.abar;
  float4 qv[NQ];
#pragma unroll
  for (int j = 0; j < NQ; ++j) {
    const int qi = q + 8 * j;
    qv[j] = qi < kq ? reinterpret_cast<const float4*>(A.q)[qi] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
  const int n_tiles = P == 0 ? 1 : (P + tile - 1) / tile;
  bool ok = true;
  m_run = -INFINITY;
  l_run = 0.0f;
#pragma unroll
  for (int j = 0; j < NV; ++j) acc[j] = make_float2(0.0f, 0.0f);
  for (int ti = 0; ti < n_tiles; ++ti) {
    const int start = ti * tile;
    const int count = max(0, min(tile, P - start));
    const bool last = ti == n_tiles - 1;
    const TileBuf tb = tile_buf(A.tiles, D, ti & 1);
    if (last) {
      // the current position as row `count` (the bulk copy writes the rows below it)
      for (int e = tid; e < kvpad; e += kThreads) {
        tb.k[count * kvpad + e] = A.kcur[e];
        tb.v[count * kvpad + e] = e < hd ? A.kv[nope + e] : 0.0f;
      }
    }
    if (count > 0) {
      if (!tile_wait(&abar[ti & 1], c.apar[ti & 1], p.timeout_ns)) {
        ok = false;
        break;
      }
      if (tid == 0) {  // every thread read the parity before the wait's barrier
        c.apar[ti & 1] ^= 1u;
        c.apend &= ~(1u << (ti & 1));
      }
    }
    if (last) __syncthreads();
    const int npos = count + (last ? 1 : 0);
    // scores: pass i covers positions 32 i + 4 w + g; after the group's butterfly, lane q keeps the
    // score of pass q (npos <= 256, so a tile has at most 8 passes)
    const int npass = (npos - 4 * warp + 31) >> 5;  // passes that hold a position of this warp (<= 0: none)
    float my_s = -INFINITY;
    for (int i = 0; i < npass; i += 2) {
      const int ka = 32 * i + 4 * warp + g, kb = ka + 32;
      float a0 = 0.0f, a1 = 0.0f, b0 = 0.0f, b1 = 0.0f;
      const float4* ra = reinterpret_cast<const float4*>(tb.k) + static_cast<size_t>(ka) * kq;
      const float4* rb = ra + 32 * kq;
#pragma unroll
      for (int j = 0; j < NQ; ++j) {
        if (q + 8 * j < kq) {
          if (ka < npos) {
            const float4 kk = ra[q + 8 * j];
            a0 = fmaf(qv[j].x, kk.x, a0);
            a1 = fmaf(qv[j].y, kk.y, a1);
            a0 = fmaf(qv[j].z, kk.z, a0);
            a1 = fmaf(qv[j].w, kk.w, a1);
          }
          if (kb < npos) {
            const float4 kk = rb[q + 8 * j];
            b0 = fmaf(qv[j].x, kk.x, b0);
            b1 = fmaf(qv[j].y, kk.y, b1);
            b0 = fmaf(qv[j].z, kk.z, b0);
            b1 = fmaf(qv[j].w, kk.w, b1);
          }
        }
      }
      float da = a0 + a1, db = b0 + b1;
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        da += __shfl_xor_sync(kFull, da, o);
        db += __shfl_xor_sync(kFull, db, o);
      }
      if (q == i && ka < npos) my_s = da;
      if (q == i + 1 && kb < npos) my_s = db;
    }
    const float m_new = fmaxf(m_run, warp_max(my_s));
    if (m_new != -INFINITY) {  // warp-uniform: the warp holds a position of this tile or an earlier one
      const float corr = m_run == -INFINITY ? 0.0f : expf(m_run - m_new);
      const float my_e = expf(my_s - m_new);  // 0 where the lane holds no position
      l_run = l_run * corr + warp_sum(my_e);
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        acc[j].x *= corr;
        acc[j].y *= corr;
      }
      // value sum: the weight of position 32 i + 4 w + gg sits in lane 8 gg + i
      const float2* V = reinterpret_cast<const float2*>(tb.v);
      for (int i = 0; i < npass; ++i) {
#pragma unroll
        for (int gg = 0; gg < 4; ++gg) {
          const float wk = __shfl_sync(kFull, my_e, 8 * gg + i);
          const int k = 32 * i + 4 * warp + gg;
          if (k < npos) {
#pragma unroll
            for (int j = 0; j < NV; ++j) {
              if (lane + 32 * j < kv2) {
                const float2 v = V[k * kv2 + lane + 32 * j];
                acc[j].x = fmaf(wk, v.x, acc[j].x);
                acc[j].y = fmaf(wk, v.y, acc[j].y);
              }
            }
          }
        }
      }
      m_run = m_new;
    }
    __syncthreads();  // the tile buffer is reused
    // each later tile refills the buffer just freed
    if (tid == 0 && ti + 2 < n_tiles)
      tile_issue(L, D, tb, h, start + 2 * tile, min(tile, P - start - 2 * tile), &abar[ti & 1], c.apend, ti & 1);
  }
  return ok;
}

// Latent attention of head h after the head's q, the latent and the head's k_rope were gathered into
// xl, in the reference decoder's form (cpu_decoder.py:186-231, ternary.cu:509-611, decoder.py:271-297):
// the latent is quantised (codes and scale appended to the compressed cache), the head's up-projection
// rows give this position's k_nope = W_k(latent) + b_k and v = W_v(latent) + b_v, the key row
// [k_nope | rotated k_rope] and the value row are appended to the head's fp32 cache, and the scaled
// query (rope pairs rotated) attends over positions 0..P with an online softmax. Cached positions
// arrive in tiles by bulk copy (double buffered); the caller issues the first two tiles before this call.
// Publishes the head's outputs. `chunk`: the op's stream chunk (the head's kv rows, a GEMV row chunk).
template <bool kTrace>
__device__ __forceinline__ bool op_attention(Ctx& c, const DecodeParams& p, const RingView& rv, const Op& opr, const IvbLayerDesc& L, int h,
                                             unsigned chunk) {
  // every field used in a loop is read once into a register: the loops store to shared memory, where
  // the context and the op record live, so reads through them would repeat
  const DecodeDims D = p.d;
  const int ll_out = opr.ll_out, kv_rows = opr.rows_per, kv_rb = opr.row_bytes, kv_ss = opr.scale_stride, kv_lg = opr.lpr_log;
  int8_t* const lat_q = L.latent_q;
  float* const lat_s = L.latent_scale;
  uint16_t* const kr_cache = L.k_rope_cache;
  float* const k_cache = L.k_cache;
  float* const v_cache = L.v_cache;
  float* const red = c.red;
  float* const stg = c.stg;
  const unsigned flag = c.flag;
  const int tid = threadIdx.x;
  const int Lt = D.latent, nope = D.nope, hd = D.head_dim, kvpad = D.kvpad;
  const int P = static_cast<int>(c.pos);
  const unsigned char* cst = stream_acquire<kAttnStages>(rv, chunk);
  bool ok = !__syncthreads_or(cst == nullptr);
  if (ok) {
    const AttnSmem A = attn_smem(c.U, D);
    const float* qh = c.xl;           // gathered q of the head
    const float* lat = c.xl + hd;     // the latent
    const float* kh = lat + Lt;       // k_rope of the head
    // the latent's codes (GEMV layout, with the half-chunk sums) and scale; the cache keeps them in order
    const float a_cur = gather_quantize_reg<4>(nullptr, Lt, flag, const_cast<float*>(lat), nullptr, 0.0f, 0.0f, D.act_eps, c.act,
                                               c.xsum, red, p.timeout_ns, nullptr);
    for (int j = tid; j < D.lpad; j += kThreads)
      lat_q[static_cast<size_t>(P) * D.lpad + j] = j < Lt ? c.act[act_slot(j)] : static_cast<int8_t>(0);
    if (tid == 0) lat_s[P] = a_cur;
    cp_async_wait_all();  // the rope row of this position
    __syncthreads();
    tick<kTrace>(c, 0);
    // k_nope and v of this position: the head's kv up-projection rows against the codes
    rows_decode(cst, kv_rows, kv_rb, kv_ss, 1, a_cur, c.act, c.xsum, Lt, kv_lg, A.kv, EPI_STORE, nullptr, nullptr, flag);
    // the scaled query (rope pairs rotated) and the rope part of this position's key (rotated, rounded
    // to fp16 as the k_rope cache holds it)
    const float scl = L.attn_scale;
    for (int e = tid; e < nope; e += kThreads) A.q[e] = qh[e] * scl;
    for (int jr = tid; jr < D.rope / 2; jr += kThreads) {
      const float cs = c.rope_s[2 * jr], sn = c.rope_s[2 * jr + 1];
      const float q0 = qh[nope + 2 * jr], q1 = qh[nope + 2 * jr + 1];
      A.q[nope + 2 * jr] = (q0 * cs - q1 * sn) * scl;
      A.q[nope + 2 * jr + 1] = (q0 * sn + q1 * cs) * scl;
      const float k0 = kh[2 * jr], k1 = kh[2 * jr + 1];
      const uint16_t r0 = f2h(k0 * cs - k1 * sn), r1 = f2h(k0 * sn + k1 * cs);
      uint16_t* kc = kr_cache + (static_cast<size_t>(h) * D.max_len + P) * D.rpad;
      kc[2 * jr] = r0;
      kc[2 * jr + 1] = r1;
      A.kcur[nope + 2 * jr] = h2f(r0);
      A.kcur[nope + 2 * jr + 1] = h2f(r1);
    }
    for (int e = hd + tid; e < kvpad; e += kThreads) {
      A.q[e] = 0.0f;
      A.kcur[e] = 0.0f;
    }
    __syncthreads();  // the kv rows are in A.kv
    for (int e = tid; e < nope; e += kThreads) A.kcur[e] = A.kv[e];
    __syncthreads();
    {
      const size_t row = (static_cast<size_t>(h) * D.max_len + P) * kvpad;
      for (int e = tid; e < kvpad; e += kThreads) {
        k_cache[row + e] = A.kcur[e];
        v_cache[row + e] = e < hd ? A.kv[nope + e] : 0.0f;
      }
    }
    tick<kTrace>(c, 1);
    float m_run, l_run;
    float2 acc[2];
    const int kq = kvpad >> 2, lane = tid & 31, warp = tid >> 5;
    if (kq <= 8) {
      float2 a1[1];
      ok = attn_tiles<1, 1>(c, p, D, L, A, h, P, m_run, l_run, a1);
      acc[0] = a1[0];
    } else if (kq <= 16) {
      float2 a1[1];
      ok = attn_tiles<2, 1>(c, p, D, L, A, h, P, m_run, l_run, a1);
      acc[0] = a1[0];
    } else {
      ok = attn_tiles<4, 2>(c, p, D, L, A, h, P, m_run, l_run, acc);
    }
    tick<kTrace>(c, 2);
    if (ok) {
      // the warps' softmax states merged: out = sum_w f_w acc_w / sum_w f_w l_w, f_w = exp(m_w - max m)
      float* const wm = red + 32;
      float* const wl = red + 40;
      if (lane == 0) {
        wm[warp] = m_run;
        wl[warp] = l_run;
      }
      for (int j = 0; j < 2; ++j)
        if (lane + 32 * j < (kvpad >> 1) && (j == 0 || kq > 16))
          reinterpret_cast<float2*>(A.part + warp * kvpad)[lane + 32 * j] = acc[j];
      __syncthreads();
      float M = wm[0];
      for (int w = 1; w < kWarps; ++w) M = fmaxf(M, wm[w]);
      for (int e = tid; e < hd; e += kThreads) {
        float num = 0.0f, den = 0.0f;
        for (int w = 0; w < kWarps; ++w) {
          const float f = wm[w] == -INFINITY ? 0.0f : expf(wm[w] - M);
          num = fmaf(f, A.part[w * kvpad + e], num);
          den = fmaf(f, wl[w], den);
        }
        stg[e] = num / den;
      }
      __syncthreads();
      ll_put(p.ll + ll_out, h * hd, stg, hd, flag);
      tick<kTrace>(c, 3);
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  if (!ok) c.fail(IVB_ETIMEOUT);
  return ok;
}

// Recurrent step of the CTA's cpc channels (one head h) after their entry rows: rows_out = [value cpc |
// gate cpc | B, C, dt of the head 3S]. Causal conv + SiLU per channel, per-state coefficients, the
// complex state update per (channel, state), the readout C.Re(state) summed over the states in order,
// skip and output gate; publishes y of the CTA's channels. Reference: ternary.cu:421-482,
// cpu_decoder.py:137-183, decoder.py:235-264.
// ssmc: [decay S | theta S | skip cpc | conv w cpc*taps | conv b cpc] from the constants chunk, then
// scratch [coef 5S | vals cpc | cpart cpc*S], then the prefetched state [cpc per state: S x cpc x 2 |
// S x cpc prev force | cpc x (taps - 1) conv window].
// float offset of the prefetched state in that region
__host__ __device__ __forceinline__ int ssm_state_off(int cpc, int S, int taps) { return 7 * S + cpc * (3 + taps) + cpc * S; }
__host__ __device__ __forceinline__ int ssm_smem_floats(int cpc, int S, int taps) {
  return 2 * S + cpc * (2 + taps) + 5 * S + cpc + cpc * S + 3 * S * cpc + cpc * (taps - 1);
}
__device__ __forceinline__ void ssm_step(Ctx& c, const DecodeParams& p, const Op& op, const IvbLayerDesc& L, const float* rows_out,
                                         float* ssmc) {
  const DecodeDims D = p.d;  // registers: the loops below store to shared memory, where p lives
  const int tid = threadIdx.x;
  const int S = D.state_dim, hd = D.head_dim, taps = D.taps, cpc = D.cpc;
  const int ch0 = c.rank * cpc, h = ch0 / hd, dd0 = ch0 - h * hd;
  const float* decay = ssmc;
  const float* theta = decay + S;
  const float* skip = theta + S;
  const float* convw = skip + cpc;
  const float* convb = convw + cpc * taps;
  float* coef = ssmc + 2 * S + cpc * (2 + taps);  // [5][S]: b, c, half_dt, a_re, a_im
  float* vals = coef + 5 * S;                    // [cpc] conv + SiLU values
  float* cpart = vals + cpc;                     // [cpc][S] readout terms
  const float* s_state = cpart + cpc * S;        // [S][cpc][2]
  const float* s_prev = s_state + 2 * S * cpc;   // [S][cpc]
  const float* s_conv = s_prev + S * cpc;        // [cpc][taps - 1]
  const float* bcdt = rows_out + 2 * cpc;
  float* const conv_state = L.conv_state;
  float2* const ssm_state = reinterpret_cast<float2*>(L.ssm_state);
  float* const prev_force = L.prev_force;
  float* const stg = c.stg;
  // the independent transcendental chains side by side, one warp each: the step coefficients of the
  // states (sigmoid -> exp, sincos), tanh of B, tanh of C, the causal conv + SiLU of the channels and
  // the output gate's sigmoid (kept in stg for the readout's thread of the same channel)
  const int warp = tid >> 5, lane = tid & 31;
  if (warp == 0) {
    for (int s2 = lane; s2 < S; s2 += 32) {
      const float half_dt = D.half_dt_min + sigmoid_f(bcdt[2 * S + s2]) * D.half_dt_range;
      const float mag = expf(2.0f * half_dt * decay[s2]);
      float sn, cs;
      sincosf(2.0f * half_dt * theta[s2], &sn, &cs);
      coef[2 * S + s2] = half_dt;
      coef[3 * S + s2] = mag * cs;
      coef[4 * S + s2] = mag * sn;
    }
  } else if (warp == 1) {
    for (int s2 = lane; s2 < S; s2 += 32) coef[s2] = tanhf(bcdt[s2]);
  } else if (warp == 2) {
    for (int s2 = lane; s2 < S; s2 += 32) coef[S + s2] = tanhf(bcdt[S + s2]);
  } else if (warp == 3) {
    for (int cl = lane; cl < cpc; cl += 32) {
      const float* win = s_conv + cl * (taps - 1);
      float* gwin = conv_state + static_cast<size_t>(ch0 + cl) * (taps - 1);
      const float incoming = rows_out[cl];
      float conv = convb[cl];
      for (int k2 = 0; k2 < taps - 1; ++k2) conv = fmaf(convw[cl * taps + k2], win[k2], conv);
      conv = fmaf(convw[cl * taps + taps - 1], incoming, conv);
      for (int k2 = 0; k2 + 1 < taps - 1; ++k2) gwin[k2] = win[k2 + 1];
      if (taps > 1) gwin[taps - 2] = incoming;
      vals[cl] = silu_f(conv);
    }
  } else if (warp == 4) {
    for (int cl = lane; cl < cpc; cl += 32) stg[cl] = sigmoid_f(rows_out[cpc + cl]);
  }
  __syncthreads();
  // one (channel, state) pair per thread: lanes run along the channels of a state (contiguous state memory)
  for (int it = tid; it < cpc * S; it += kThreads) {
    const int s2 = it / cpc, cl = it - s2 * cpc;
    const int li = s2 * cpc + cl;
    const size_t gi = static_cast<size_t>(h * S + s2) * hd + dd0 + cl;
    const float b = coef[s2], cc = coef[S + s2], half_dt = coef[2 * S + s2];
    const float ar = coef[3 * S + s2], ai = coef[4 * S + s2];
    const float prev = s_prev[li];
    const float sr = s_state[2 * li], si = s_state[2 * li + 1];
    const float force = b * vals[cl];
    const float dr = (force + ar * prev) * half_dt;
    const float di = (ai * prev) * half_dt;
    const float nr = sr * ar - si * ai + dr;
    const float ni = sr * ai + si * ar + di;
    ssm_state[gi] = make_float2(nr, ni);
    prev_force[gi] = force;
    cpart[cl * S + s2] = cc * nr;
  }
  __syncthreads();
  for (int cl = tid; cl < cpc; cl += kThreads) {
    float contrib = 0.0f;
    const float* cp = cpart + cl * S;
    if ((S & 3) == 0 && (reinterpret_cast<uintptr_t>(cp) & 15) == 0) {
#pragma unroll 4
      for (int s4 = 0; s4 < S; s4 += 4) {  // independent 16-byte loads; the sum stays in state order
        const float4 v = *reinterpret_cast<const float4*>(cp + s4);
        contrib += v.x;
        contrib += v.y;
        contrib += v.z;
        contrib += v.w;
      }
    } else {
      for (int s2 = 0; s2 < S; ++s2) contrib += cp[s2];
    }
    // published by the thread that computed it (its gate sigmoid is in stg[cl])
    ll_store(p.ll + op.ll_out + ch0 + cl, __float_as_uint((contrib + skip[cl] * vals[cl]) * stg[cl]), c.flag);
  }
}

// Local top-k of the head op: keys[0, n) (n <= 256, one per thread) ranked by (key desc, index asc);
// those of rank < k go to out_key/out_id in order. Every thread counts the keys above its own.
static __device__ __noinline__ void topk_by_rank(const unsigned* keys, int n, int k, int id_base, unsigned* out_key, int* out_id) {
  const int tid = threadIdx.x;
  if (tid < n) {
    const unsigned mine = keys[tid];
    int rank = 0;
    for (int o = 0; o < n; ++o) {
      const unsigned ko = keys[o];
      rank += (ko > mine || (ko == mine && o < tid)) ? 1 : 0;
    }
    if (rank < k) {
      out_key[rank] = mine;
      out_id[rank] = id_base + tid;
    }
  }
  __syncthreads();
}

// Every GEMV op (entry projections, out, gate/up, down, head) of one CTA: prefetches for the op's
// epilogue, the gathered and (normed) quantised input, its rows chunk by chunk from the weight ring,
// and the epilogue (publish the output slice, residual add, SwiGLU, the recurrent step, or the head's
// logits and local top-k candidates).
template <bool kTrace>
__device__ __forceinline__ bool op_gemv(Ctx& c, const DecodeParams& p, const RingView& rv, const Op& opr, const IvbLayerDesc& lay,
                                        int rows_c) {
  // the op record, the dimensions and the context fields used below are read once into registers (the
  // op stores to shared memory, where all three live)
  const Op op = opr;
  unsigned idx = c.chunk_base + op.first_chunk;  // the op's chunks: [norm] [constants] rows...
  const DecodeDims D = p.d;
  unsigned char* U = c.U;
  const int tid = threadIdx.x;
  const unsigned flag = c.flag;
  const int lo = min(op.rows_total, static_cast<int>(c.rank) * op.rows_per);
  float* rows_out = c.loc;
  bool ok = true;
  const unsigned char* cst = nullptr;
  float* ssmc = reinterpret_cast<float*>(U);
  const int S = D.state_dim, taps = D.taps, cpc = D.cpc;
  if (op.kind == OP_HEAD && c.sampling && ((lo | rows_c) & 3) == 0) {
    // the repetition flags of my vocabulary slice, for the local top-k
    const float* src = reinterpret_cast<const float*>(p.seen + lo);
    for (int i = tid; i < rows_c / 4; i += kThreads) cp_async_f32(c.seen_s + i, src + i);
    cp_async_commit();
  } else if (op.kind == OP_ENTRY_MAMBA) {
    // the recurrent state of my channels streams into shared memory while the rows are computed:
    // per state s the cpc complex values and previous forces of my channels, then the conv windows
    const int hd = D.head_dim, ch0 = c.rank * cpc;
    float* dst = ssmc + ssm_state_off(cpc, S, taps);
    if (D.ssm_v16) {
      // one 16-byte copy per thread, indices by shifts: per state cpc / 2 chunks of complex values and
      // cpc / 4 of previous forces, then the conv windows (every piece 16-byte aligned, checked on the host)
      const int lg = D.ssm_lg_cs, cs = 1 << lg, n0 = S << lg, n1 = S << (lg - 1), n2 = (cpc * (taps - 1)) >> 2;
      const int row0 = c.ssm_row0;
      const int j = tid;
      if (j < n0 + n1 + n2) {
        const float* src;
        float* d2;
        if (j < n0) {
          const int s2 = j >> lg, r = j & (cs - 1);
          src = lay.ssm_state + static_cast<size_t>(row0 + s2 * hd) * 2 + 4 * r;
          d2 = dst + 2 * cpc * s2 + 4 * r;
        } else if (j < n0 + n1) {
          const int jj = j - n0, s2 = jj >> (lg - 1), r = jj & ((cs >> 1) - 1);
          src = lay.prev_force + static_cast<size_t>(row0 + s2 * hd) + 4 * r;
          d2 = dst + 2 * S * cpc + cpc * s2 + 4 * r;
        } else {
          const int jj = j - n0 - n1;
          src = lay.conv_state + static_cast<size_t>(ch0) * (taps - 1) + 4 * jj;
          d2 = dst + 3 * S * cpc + 4 * jj;
        }
        cp_async_16(d2, src);
      }
      cp_async_commit();
    } else {
      const int h = ch0 / hd, dd0 = ch0 - h * hd;
      const int l0 = 2 * S * cpc, l1 = S * cpc, l2 = cpc * (taps - 1);
      for (int i = tid; i < l0 + l1 + l2; i += kThreads) {
        const float* src;
        if (i < l0) {
          const int s2 = i / (2 * cpc), r = i - s2 * 2 * cpc;
          src = lay.ssm_state + (static_cast<size_t>(h * S + s2) * hd + dd0) * 2 + r;
        } else if (i < l0 + l1) {
          const int s2 = (i - l0) / cpc, r = (i - l0) - s2 * cpc;
          src = lay.prev_force + static_cast<size_t>(h * S + s2) * hd + dd0 + r;
        } else {
          src = lay.conv_state + static_cast<size_t>(ch0) * (taps - 1) + (i - l0 - l1);
        }
        cp_async_f32(dst + i, src);
      }
      cp_async_commit();
    }
  }
  tick<kTrace>(c, 0);
  // the input: the previous op's output gathered from its flag words (or the embedding / combined
  // attention already in shared memory), normed with the weights of its own stream chunk, quantised
  const unsigned char* nrm = nullptr;
  if (op.has_norm_chunk) {
    nrm = stream_acquire(rv, idx++);
    if (nrm == nullptr) ok = false;
  }
  const bool from_smem = op.ll_in < 0;
  float* keep = op.in_dst == IN_RESID ? c.resid : nullptr;  // the residual replica; other inputs live in registers only
  long long* t_arr = kTrace && c.marks != nullptr ? &c.prof_t2 : nullptr;
  const unsigned long long* src = from_smem ? nullptr : p.ll + op.ll_in;
  const float* nw = op.has_norm ? reinterpret_cast<const float*>(nrm) : nullptr;
  const float act_scale =
      op.in_n <= 4 * kThreads
          ? gather_quantize_reg<4>(src, op.in_n, flag, keep, nw, op.norm_eps, D.clip, D.act_eps, c.act, c.xsum, c.red, p.timeout_ns, t_arr)
          : gather_quantize_reg<kMaxEPT>(src, op.in_n, flag, keep, nw, op.norm_eps, D.clip, D.act_eps, c.act, c.xsum, c.red, p.timeout_ns,
                                         t_arr);
  if (act_scale < 0.0f) ok = false;
  if (kTrace && tid == 0 && c.marks != nullptr && !from_smem) {  // split the wait for the input from the quantiser
    c.prof[1] += c.prof_t2 - c.prof_t;
    c.prof_t = c.prof_t2;
  }
  if (op.has_const) {
    cst = stream_acquire(rv, idx++);
    if (cst == nullptr) ok = false;
  }
  tick<kTrace>(c, 2);
  // SSM constants leave the stage before it is recycled
  if (op.kind == OP_ENTRY_MAMBA && cst != nullptr) {
    const int e0 = S, e1 = 2 * S, e2 = e1 + cpc, e3 = e2 + cpc * taps, e4 = e3 + cpc;
    for (int i = tid; i < e4; i += kThreads) {
      const float* src = i < e0   ? reinterpret_cast<const float*>(cst + op.c_decay) + i
                         : i < e1 ? reinterpret_cast<const float*>(cst + op.c_theta) + (i - e0)
                         : i < e2 ? reinterpret_cast<const float*>(cst + op.c_skip) + (i - e1)
                         : i < e3 ? reinterpret_cast<const float*>(cst + op.c_convw) + (i - e2)
                                  : reinterpret_cast<const float*>(cst + op.c_convb) + (i - e3);
      ssmc[i] = *src;
    }
  }
  // rows of this CTA, chunk by chunk (a warp skips a chunk whose wait ran out in any of its lanes); the
  // out, down, gate/up and mla entry projections publish each row as it finishes
  const int epi = op.kind == OP_OUT || op.kind == OP_DOWN           ? EPI_RESID
                  : op.kind == OP_GATE_UP && op.lpr_log <= 4          ? EPI_SWIGLU
                  : op.kind == OP_ENTRY_MLA                           ? EPI_PUBLISH
                                                                      : EPI_STORE;
  unsigned long long* const ll_out = p.ll + op.ll_out + (epi == EPI_SWIGLU ? lo / 2 : lo);
  const float* const resid = c.resid + lo;
  const int n_row_chunks = op.n_chunks - op.has_const - op.has_norm_chunk;
  for (int ch = 0; ch < n_row_chunks; ++ch) {
    const unsigned char* stage = stream_acquire(rv, idx++);
    if (!__all_sync(kFull, stage != nullptr)) {
      ok = false;
    } else {
      const int r0 = ch * op.chunk_rows;
      const int k = max(0, min(op.chunk_rows, rows_c - r0));
      if (k > 0)
        rows_decode(stage, k, op.row_bytes, op.scale_stride, op.has_bias, act_scale, c.act, c.xsum, op.in_n, op.lpr_log,
                    rows_out + r0, epi, ll_out + (epi == EPI_SWIGLU ? r0 / 2 : r0), resid + r0, flag);
    }
  }
  if (epi == EPI_STORE) __syncthreads();  // every row of this CTA is in rows_out
  tick<kTrace>(c, 3);
  float* stg = c.stg;
  // epilogues that need every row of the CTA
  if (op.kind == OP_GATE_UP && epi == EPI_STORE) {
    for (int m = tid; m < rows_c / 2; m += kThreads) stg[m] = silu_f(rows_out[2 * m]) * rows_out[2 * m + 1];
    __syncthreads();
    ll_put(p.ll + op.ll_out, lo / 2, stg, rows_c / 2, flag);
  } else if (op.kind == OP_HEAD) {
    for (int r = tid; r < rows_c; r += kThreads) p.logits[lo + r] = rows_out[r];
    if (c.sampling) {
      // local top-k of my vocabulary slice (rows_c <= 256, one key per thread) for the sampler
      unsigned* keys = reinterpret_cast<unsigned*>(U);
      unsigned* ok_key = keys + kThreads;
      int* ok_id = reinterpret_cast<int*>(ok_key + p.kc);
      cp_async_wait_all();
      __syncthreads();
      const uint8_t* seen_b = reinterpret_cast<const uint8_t*>(c.seen_s);
      const bool pref = ((lo | rows_c) & 3) == 0;
      for (int r = tid; r < rows_c; r += kThreads)
        keys[r] = score_key(rows_out[r], pref ? seen_b[r] : __ldcg(p.seen + lo + r), c.inv_t, c.pen, c.ipen);
      __syncthreads();
      const int kl = min(c.K, rows_c);
      topk_by_rank(keys, rows_c, kl, lo, ok_key, ok_id);
      const int R = D.R, kp = c.kp;
      cand_put(p.ll + op.ll_out + static_cast<size_t>(c.rank) * kp, p.ll + op.ll_out + static_cast<size_t>(R) * kp + static_cast<size_t>(c.rank) * kp,
               ok_key, ok_id, kl, kp, 0x40000000u + c.rank * static_cast<unsigned>(kp), flag);
    }
  } else if (op.kind == OP_ENTRY_MAMBA) {
    cp_async_wait_all();
    __syncthreads();
    ssm_step(c, p, opr, lay, rows_out, ssmc);
  }
  tick<kTrace>(c, 4);
  if (!ok) atomicCAS(p.error, 0u, static_cast<unsigned>(IVB_ETIMEOUT));
  return ok;
}

// Group leaders (two-level merges only): the top-k of their group's head candidates, published as kq slots.
static __device__ __noinline__ bool op_merge(Ctx& c, const Op& op) {
  const DecodeParams& p = *c.p;
  const DecodeDims& D = p.d;
  const int R = D.R;
  if (!c.sampling || !c.two_level || c.rank % D.group != 0) return true;  // candidates exist only when sampling
  const int g = c.rank / D.group;
  const int nblk = min(D.group, R - g * D.group);
  const int kp = c.kp, kq = c.kq;
  const unsigned long long* hbuf = p.ll + op.ll_in;
  unsigned* mk = reinterpret_cast<unsigned*>(c.U + p.sm.cand);
  int* mi = reinterpret_cast<int*>(mk + nblk * kp);
  unsigned* ck = reinterpret_cast<unsigned*>(c.U);
  int* ci = reinterpret_cast<int*>(ck + p.kc);
  unsigned* sk = reinterpret_cast<unsigned*>(ci + p.kc);
  int* si = reinterpret_cast<int*>(sk + p.kc);
  TopkScratch ts{reinterpret_cast<unsigned*>(si + p.kc), reinterpret_cast<int*>(si + p.kc) + kWarps * 256};
  const size_t first = static_cast<size_t>(g) * D.group * kp;
  if (!ll_gather2(hbuf + first, nblk * kp, hbuf + static_cast<size_t>(R) * kp + first, nblk * kp, c.flag, mk, p.timeout_ns)) {
    c.fail(IVB_ETIMEOUT);
    return false;
  }
  const int kk = min(c.K, nblk * kp);
  topk_sorted(mk, mi, 0, nblk * kp, kk, ts, ck, ci, sk, si);
  cand_put(p.ll + op.ll_out + static_cast<size_t>(g) * kq, p.ll + op.ll_out + static_cast<size_t>(c.n_groups) * kq + static_cast<size_t>(g) * kq,
           sk, si, kk, kq, 0x60000000u + static_cast<unsigned>(g * kq), c.flag);
  return true;
}

// Every CTA: merge the candidates (of the group leaders, or of every head CTA) and draw the same token
// with the Philox uniform of counter rctr. Returns the token, or -1 when a wait ran out.
static __device__ __noinline__ int draw_next(Ctx& c, uint64_t rkey, uint64_t rctr) {
  const DecodeParams& p = *c.p;
  const int kc = p.kc, R = p.d.R;
  const int nblk = c.two_level ? c.n_groups : R;
  const int kb = c.two_level ? c.kq : c.kp;
  const unsigned long long* src = p.ll + (c.two_level ? p.ops[p.n_ops - 1].op.ll_out : p.ops[p.head_op].op.ll_out);
  unsigned* mk = reinterpret_cast<unsigned*>(c.U + p.sm.cand);
  int* mi = reinterpret_cast<int*>(mk + nblk * kb);
  unsigned* ck = reinterpret_cast<unsigned*>(c.U);
  int* ci = reinterpret_cast<int*>(ck + kc);
  unsigned* sk = reinterpret_cast<unsigned*>(ci + kc);
  int* si = reinterpret_cast<int*>(sk + kc);
  float* cdf = reinterpret_cast<float*>(si + kc);
  TopkScratch ts{reinterpret_cast<unsigned*>(cdf + kc), reinterpret_cast<int*>(cdf + kc) + kWarps * 256};
  if (!ll_gather(src, nblk * 2 * kb, c.flag, mk, p.timeout_ns)) {
    c.fail(IVB_ETIMEOUT);
    return -1;
  }
  const int n = nblk * kb;
  const int kk = min(c.K, n);
  topk_sorted(mk, mi, 0, n, kk, ts, ck, ci, sk, si);
  return draw_token(sk, si, kk, cdf, c.red, rkey, rctr);
}

template <bool kTrace>
__global__ void __launch_bounds__(kThreads, 1) grid_decode_kernel(const __grid_constant__ DecodeParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) unsigned long long full[kStages];
  __shared__ __align__(8) unsigned long long abar[2];
  __shared__ __align__(16) OpRec opbuf[2];  // the running op and the next one (descriptor + layer)
  __shared__ __align__(16) int rowsbuf[2][4];
  __shared__ Ctx c;
  __shared__ Stream st;
  __shared__ __align__(16) DecodeParams ps;  // the parameters, read by the op routines from shared memory
  const unsigned rank = blockIdx.x;
  const int tid = threadIdx.x;
  const DecodeDims& D = p.d;
  const DecodeSmem& M = p.sm;
  const int R = D.R;
  const bool attn_cta = static_cast<int>(rank) >= R;  // one per head: runs only the attention ops
  const int cpt = attn_cta ? p.n_mla : p.chunks_per_token;
  const unsigned long long* my_addr =
      attn_cta ? p.attn_addr + static_cast<size_t>(rank - R) * p.n_mla : p.chunk_addr + static_cast<size_t>(rank) * cpt;
  const unsigned* my_bytes =
      attn_cta ? p.attn_bytes + static_cast<size_t>(rank - R) * p.n_mla : p.chunk_bytes + static_cast<size_t>(rank) * cpt;
  unsigned long long* caddr = reinterpret_cast<unsigned long long*>(smem + M.ctab);
  unsigned* cbytes = reinterpret_cast<unsigned*>(caddr + p.chunks_per_token);
  for (int k = tid; k < cpt; k += kThreads) {
    caddr[k] = my_addr[k];
    cbytes[k] = my_bytes[k];
  }
  for (int i = tid; i < static_cast<int>(sizeof(DecodeParams) / 4); i += kThreads)
    reinterpret_cast<unsigned*>(&ps)[i] = reinterpret_cast<const unsigned*>(&p)[i];
  // op descriptors travel through a two-slot shared buffer: op k+1 is fetched while op k runs
  auto fetch_op = [&](int oi, int slot) {
    if (tid < static_cast<int>(sizeof(OpRec) / 16))
      cp_async_16(reinterpret_cast<unsigned char*>(&opbuf[slot]) + 16 * tid,
                  reinterpret_cast<const unsigned char*>(p.ops + oi) + 16 * tid);
    else if (tid == kThreads - 1 && !attn_cta)
      cp_async_f32(reinterpret_cast<float*>(&rowsbuf[slot][0]), reinterpret_cast<const float*>(p.op_rows + oi * R + rank));
    cp_async_commit();
  };
  fetch_op(attn_cta ? (p.n_mla > 0 ? p.attn_ops[0] : 0) : 0, 0);
  long long tok = p.feed != nullptr ? ldcg_i64(p.feed) : ldcg_i64(p.token);
  const unsigned epoch0 = __ldcg(p.epoch);
  const uint64_t rkey = p.rng[0];
  uint64_t rctr = p.rng[1];
  if (tid == 0) {
    for (int s2 = 0; s2 < kStages; ++s2) mbar_init(&full[s2], 1);
    mbar_init(&abar[0], 1);
    mbar_init(&abar[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    st.full = full;
    // an attention CTA streams through the ring's last kAttnStages stages; the rest of the ring extends
    // its attention tiles
    st.ring = smem + M.ring + (attn_cta ? (kStages - kAttnStages) * M.stage_bytes : 0);
    st.stage_bytes = M.stage_bytes;
    st.caddr = caddr;
    st.cbytes = cbytes;
    st.cpt = cpt;
    st.head_first = attn_cta ? cpt : p.head_first;  // the attention CTAs' chunks never belong to a head
    st.issued = 0u;
    st.p_step = 0;
    st.p_chunk = 0;
    c.p = &ps;
    c.st = &st;
    c.chunk_base = 0u;
    c.rank = rank;
    c.resid = reinterpret_cast<float*>(smem + M.resid);
    c.loc = reinterpret_cast<float*>(smem + M.loc);
    c.red = reinterpret_cast<float*>(smem + M.red);
    c.xl = reinterpret_cast<float*>(smem + M.xl);
    c.stg = reinterpret_cast<float*>(smem + M.pub);  // this op's output slice before it is published
    c.rope_s = reinterpret_cast<float*>(smem + M.rope_row);
    c.seen_s = reinterpret_cast<float*>(smem + M.seen);  // bytes; float* for the 4-byte copies
    c.act = reinterpret_cast<int8_t*>(smem + M.act);
    c.xsum = reinterpret_cast<int*>(smem + M.xsum);
    c.U = smem + M.u;
    c.abar = abar;
    c.apar[0] = c.apar[1] = 0u;
    c.apend = 0u;
    {
      const int ch0 = static_cast<int>(rank) * D.cpc, h = ch0 / D.head_dim;
      c.ssm_row0 = h * D.state_dim * D.head_dim + (ch0 - h * D.head_dim);
    }
    c.marks = nullptr;
    c.pos = ldcg_i64(p.position);
    c.inv_t = 1.0f / __ldcg(p.sampling);
    c.pen = __ldcg(p.sampling + 1);
    c.ipen = __ldcg(p.sampling + 2);
    c.sampling = (p.flags & IVB_RUN_SAMPLE) != 0;
    const long long kreq = ldcg_i64(p.top_k);
    const int cap = min(min(D.max_top_k, D.vocab), kMaxTopK);
    c.K = static_cast<int>(kreq < 1 ? 1 : (kreq > cap ? cap : kreq));
    // candidate layout of this run (uniform across the CTAs): kp slots per GEMV CTA; when they do not
    // all fit one merge, group leaders first reduce their groups to kq slots each
    c.kp = cand_slots(c.K, p.ops[p.head_op].op.rows_per);
    c.n_groups = (R + D.group - 1) / D.group;
    c.two_level = c.n_groups > 1 && R * c.kp > D.cand_cap;
    c.kq = (min(c.K, D.group * c.kp) + 1) & ~1;
    if (attn_cta) stream_refill<kAttnStages>(p, &st, 0u);
    else stream_refill(p, &st, 0u);
  }
  cp_async_wait_all();
  __syncthreads();
  // the ring as its consumers see it (an attention CTA streams through the last kAttnStages stages)
  const RingView rv{full, smem + M.ring + (attn_cta ? (kStages - kAttnStages) * M.stage_bytes : 0), M.stage_bytes, p.timeout_ns};
  unsigned opk = 0;  // ops run so far (selects the descriptor slot)
  bool alive = true;
  if (attn_cta) {
    // ---------------- attention CTA of head h: the attention op of every mla block ----------------
    const int h = static_cast<int>(rank) - R;
    for (int step = 0; step < p.steps && alive; ++step) {
      const long long pos = c.pos;
      if (pos < 0 || pos >= D.max_len) break;  // GEMV CTA 0 reports it
      const unsigned flag = epoch0 + static_cast<unsigned>(step) + 1u;
      const bool tracing = p.trace != nullptr && step == p.trace_step;
      if (tid == 0) c.flag = flag;
      for (int mi = 0; mi < p.n_mla && alive; ++mi) {
        const int oi = p.attn_ops[mi];
        const Op& op = opbuf[opk & 1].op;
        const IvbLayerDesc& lay = opbuf[opk & 1].layer;
        fetch_op(p.attn_ops[mi + 1 < p.n_mla ? mi + 1 : 0], (opk + 1) & 1);
        if (kTrace && tid == 0) {
          c.marks = tracing ? p.trace + (static_cast<size_t>(oi) * (R + D.A) + rank) * 8 : nullptr;
          for (int k = 0; k < 6; ++k) c.prof[k] = 0;
          c.prof_t = c.marks != nullptr ? clock64() : 0;
          mark(c.marks, 0);
        }
        // the first two tiles of cached positions (independent of this token) before the input arrives
        if (tid == 0 && pos > 0) {
          const int np = static_cast<int>(pos);
          unsigned char* tiles = attn_smem(c.U, D).tiles;
          tile_issue(lay, D, tile_buf(tiles, D, 0), h, 0, min(np, D.tile), &abar[0], c.apend, 0);
          if (np > D.tile) tile_issue(lay, D, tile_buf(tiles, D, 1), h, D.tile, min(np - D.tile, D.tile), &abar[1], c.apend, 1);
        }
        // the rope row of this position (waited for inside), and the head's q, the latent and the
        // head's k_rope from the entry op's output [q | latent | k_rope]
        const float* rrow = lay.rope + static_cast<size_t>(pos) * D.rope;
        for (int i = tid; i < D.rope; i += kThreads) cp_async_f32(c.rope_s + i, rrow + i);
        cp_async_commit();
        const unsigned long long* src = p.ll + op.ll_in;
        bool ok = ll_gather3(src + h * D.head_dim, D.head_dim, src + D.hidden, D.latent, src + D.hidden + D.latent + h * D.rope,
                             D.rope, flag, reinterpret_cast<unsigned*>(c.xl), p.timeout_ns);
        tick<kTrace>(c, 5);
        const unsigned chunk = c.chunk_base + static_cast<unsigned>(mi);
        if (ok) ok = op_attention<kTrace>(c, p, rv, op, lay, h, chunk);
        else c.fail(IVB_ETIMEOUT);
        if (kTrace && tid == 0 && c.marks != nullptr) {
          for (int k = 0; k < 6; ++k) c.marks[1 + k] = static_cast<unsigned long long>(c.prof[k]);
          mark(c.marks, 7);
        }
        if (!ok && tid == 0) attn_drain(c, p.timeout_ns);  // tile copies a failed op left in flight
        cp_async_wait_all();
        ++opk;
        const bool failed = __syncthreads_or(!ok);
        if (tid == 0) stream_refill<kAttnStages>(p, &st, chunk + 1);
        if (failed) alive = false;
      }
      if (tid == 0) {
        c.pos = pos + 1;
        c.chunk_base += static_cast<unsigned>(p.n_mla);
      }
      __syncthreads();
    }
  } else {
    // ---------------- GEMV CTA: every projection op of the token program ----------------
    for (int step = 0; step < p.steps && alive; ++step) {
      if (step > 0 && p.feed != nullptr) tok = ldcg_i64(p.feed + step);
      const long long pos = c.pos;
      if (pos < 0 || pos >= D.max_len || tok < 0 || tok >= D.vocab) {
        // every CTA sees the same values: stop together
        if (rank == 0 && tid == 0) atomicCAS(p.error, 0u, static_cast<unsigned>(pos >= D.max_len ? IVB_ECAPACITY : IVB_EINVAL));
        break;
      }
      const bool head = head_needed(p, step);
      const bool tracing = p.trace != nullptr && step == p.trace_step;
      if (tid == 0) c.flag = epoch0 + static_cast<unsigned>(step) + 1u;
      // embedding of the token -> residual replica (every GEMV CTA computes the whole row)
      {
        const uint8_t* erow = p.head.packed + static_cast<size_t>(tok) * p.head.row_bytes;
        const uint16_t* srow = p.head.scales + static_cast<size_t>(tok) * p.head.scale_stride;
        float* resid = reinterpret_cast<float*>(smem + M.resid);
        for (int i = tid; i < D.hidden; i += kThreads)
          resid[i] = static_cast<float>(((__ldg(erow + (i >> 2)) >> ((i & 3) << 1)) & 3) - 1) * h2f(__ldg(srow + (i >> 7)));
      }
      __syncthreads();
      const int n_run = head ? p.n_ops : p.head_op;  // the head (and the candidate merge) end the program
      for (int oi = 0; oi < n_run && alive; ++oi) {
        const Op& op = opbuf[opk & 1].op;  // fields are read from shared memory where used
        const IvbLayerDesc& lay = opbuf[opk & 1].layer;
        const int rows_c = rowsbuf[opk & 1][0];
        fetch_op(oi + 1 < n_run ? oi + 1 : 0, (opk + 1) & 1);  // the op after this one (op 0 of the next token)
        if (kTrace && tid == 0) {
          c.marks = tracing && op.kind != OP_ATTN ? p.trace + (static_cast<size_t>(oi) * (R + D.A) + rank) * 8 : nullptr;
          for (int k = 0; k < 6; ++k) c.prof[k] = 0;
          c.prof_t = c.marks != nullptr ? clock64() : 0;
          mark(c.marks, 0);
        }
        bool ok = true;
        if (op.kind == OP_MERGE) {
          ok = op_merge(c, op);
        } else if (op.kind != OP_ATTN) {  // the attention CTAs run the attention ops
          ok = op_gemv<kTrace>(c, p, rv, op, lay, rows_c);
        }
        tick<kTrace>(c, 5);
        if (kTrace && tid == 0 && c.marks != nullptr) {
          for (int k = 0; k < 6; ++k) c.marks[1 + k] = static_cast<unsigned long long>(c.prof[k]);
          mark(c.marks, 7);
        }
        cp_async_wait_all();  // the next descriptor has landed
        ++opk;
        // local buffers (rows, codes, staging) are reused by the next op, and the op's ring stages are free
        const bool failed = __syncthreads_or(!ok);
        if (tid == 0) stream_refill(p, &st, c.chunk_base + op.first_chunk + op.n_chunks);
        if (failed) {
          alive = false;
          break;
        }
      }
      if (!alive) break;
      if (c.sampling) {
        const int chosen = draw_next(c, rkey, rctr);
        if (chosen < 0) break;
        ++rctr;
        tok = chosen;
        if (tid == 0) {
          // the CTA whose vocabulary slice holds the token sets its flag (it alone reads that slice)
          const int per = p.ops[p.head_op].op.rows_per;
          if (chosen / per == static_cast<int>(rank)) p.seen[chosen] = 1;
          if (rank == 0) {
            p.token[0] = chosen;
            p.rng[1] = rctr;
            if (p.history != nullptr && step < p.history_len) p.history[step] = chosen;
          }
        }
      }
      if (tid == 0) {
        c.pos = pos + 1;
        c.chunk_base += static_cast<unsigned>(chunks_of_step(p, &st, step));
        if (rank == 0) p.position[0] = pos + 1;
      }
      __syncthreads();
    }
    // every flag of this run is at most epoch0 + steps: the next run starts above it
    if (rank == 0 && tid == 0) *p.epoch = epoch0 + static_cast<unsigned>(p.steps);
  }
  // let every in-flight copy land before the CTA's shared memory goes away: the descriptor prefetch,
  // and the ring (at most the last ns chunks issued can still be in flight)
  cp_async_wait_all();
  if (tid == 0) {
    const unsigned issued = st.issued;
    const unsigned ns = attn_cta ? kAttnStages : kStages;
    for (unsigned k = issued > ns ? issued - ns : 0u; k < issued; ++k)
      if (!mbar_wait_bounded(full + k % ns, (k / ns) & 1u, p.timeout_ns)) break;
  }
  __syncthreads();
}

// Unit probe of the decode kernel's row routine: the stage (one stream chunk, k rows) goes to shared
// memory, the int8 codes into the transposed GEMV layout with their half-chunk sums (what the quantiser
// of the decode kernel writes), then rows_generic with 2^lg lanes per row stores the k row values.
__global__ void __launch_bounds__(kThreads, 1) rows_probe_kernel(const unsigned char* stage, int stage_bytes, int k, int row_bytes,
                                                                 int sstride, int has_bias, float act_scale, const int8_t* q8,
                                                                 int in_n, int lg, float* out) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int padded = (in_n + 63) & ~63, chunks = padded >> 6;
  unsigned char* st = smem;
  int8_t* act = reinterpret_cast<int8_t*>(smem + round16(stage_bytes));
  int* xhalf = reinterpret_cast<int*>(act + padded);
  float* res = reinterpret_cast<float*>(xhalf + 2 * chunks);
  for (int i = threadIdx.x; i < stage_bytes; i += kThreads) st[i] = stage[i];
  for (int i = threadIdx.x; i < padded; i += kThreads) act[act_slot(i)] = i < in_n ? q8[i] : static_cast<int8_t>(0);
  for (int h = threadIdx.x; h < 2 * chunks; h += kThreads) {
    int sum = 0;
    for (int i = 32 * h; i < 32 * h + 32; ++i) sum += i < in_n ? q8[i] : 0;
    xhalf[h] = sum;
  }
  __syncthreads();
  if (lg < 0) rows_decode(st, k, row_bytes, sstride, has_bias, act_scale, act, xhalf, in_n, 4, res, EPI_STORE, nullptr, nullptr, 0u);
  else rows_generic(st, k, row_bytes, sstride, has_bias, act_scale, act, xhalf, in_n, lg, res, EPI_STORE, nullptr, nullptr, 0u);
  __syncthreads();
  for (int r = threadIdx.x; r < k; r += kThreads) out[r] = res[r];
}

}  // namespace ivb

// ------------------------------------------------------------------------------------------------
// host plan: per-CTA weight streams, op program, flag-word buffers, shared-memory map
// ------------------------------------------------------------------------------------------------
namespace {

struct CopyOp {       // one device-to-device copy into the stream, executed at bind
  size_t dst;         // byte offset in the stream
  const void* src;    // nullptr: zero fill
  size_t width;       // bytes per row
  size_t rows;
  size_t spitch, dpitch;
};

struct Segment {      // rows [row0, row0 + count) of one matrix
  const IvbTernary* m;
  int row0, count;
};

size_t r16(size_t v) { return (v + 15) / 16 * 16; }

}  // namespace

struct IvbDecoder {
  IvbModelDesc desc;
  std::vector<IvbLayerDesc> layers;
  ivb::DecodeDims d;
  ivb::DecodeSmem sm;
  std::vector<ivb::Op> ops;
  std::vector<ivb::OpRec> recs;  // device op records, kept alive until the upload completes
  std::vector<int32_t> op_rows;
  std::vector<unsigned long long> chunk_off;  // byte offset into the stream blob, or ~0 for a pointer chunk
  std::vector<unsigned long long> chunk_ptr;  // device address of a pointer chunk (a shared array read in place)
  std::vector<unsigned long long> chunk_addr; // device addresses (filled at bind)
  std::vector<unsigned> chunk_bytes;
  std::vector<unsigned long long> attn_off;   // [A][n_mla] blob offsets of the attention CTAs' chunks
  std::vector<unsigned long long> attn_addr;  // device addresses (filled at bind)
  std::vector<unsigned> attn_bytes;
  std::vector<int32_t> attn_ops;              // indices of the attention ops
  std::vector<CopyOp> copies;
  int32_t R, A, cpt, head_first, head_op, kc;
  size_t stream_bytes, smem, ll_words;
  size_t off_stream, off_ops, off_op_rows, off_chunk_addr, off_chunk_bytes, off_attn_addr, off_attn_bytes, off_attn_ops, off_ll,
      off_sync, total;
  unsigned char* ws;
  unsigned long long* trace;
  int32_t trace_step;
};

namespace ivb {

static int32_t validate(const IvbModelDesc& d) {
  if (d.abi_version != IVB_ABI_VERSION) return fail(IVB_EINVAL, "abi_version %d != %d", d.abi_version, IVB_ABI_VERSION);
  if (d.vocab <= 0 || d.hidden <= 0 || d.heads <= 0 || d.num_layers <= 0 || d.max_len <= 0 || d.dense <= 0)
    return fail(IVB_EINVAL, "model dimensions must be positive");
  if (d.hidden % d.heads != 0 || d.head_dim * d.heads != d.hidden) return fail(IVB_EINVAL, "hidden must equal heads * head_dim");
  if (d.state_dim > kMaxStateDim) return fail(IVB_EINVAL, "state_dim %d > %d", d.state_dim, kMaxStateDim);
  if (d.latent_dim > 32 * kMaxLatentPerLane) return fail(IVB_EINVAL, "latent_dim %d > %d", d.latent_dim, 32 * kMaxLatentPerLane);
  if (d.rope_dim + d.nope_dim != d.head_dim || (d.rope_dim & 1)) return fail(IVB_EINVAL, "rope_dim + nope_dim must equal head_dim");
  if ((d.head_dim & 1) || (d.latent_dim & 1)) return fail(IVB_EINVAL, "head_dim and latent_dim must be even");
  if (d.head_dim > 128) return fail(IVB_EINVAL, "head_dim %d > 128", d.head_dim);
  if (d.max_top_k <= 0) return fail(IVB_EINVAL, "max_top_k must be positive");
  if (!d.layers || !d.logits || !d.token || !d.position || !d.seen || !d.sampling || !d.top_k || !d.rng || !d.final_norm)
    return fail(IVB_EINVAL, "null state pointer in the model description");
  if (int32_t rc = check_ternary(d.head, "head")) return rc;
  if (d.head.rows != d.vocab || d.head.in_features != d.hidden) return fail(IVB_EINVAL, "head must be [vocab, hidden]");
  int taps = -1;
  for (int i = 0; i < d.num_layers; ++i) {
    const IvbLayerDesc& L = d.layers[i];
    char name[64];
    snprintf(name, sizeof(name), "layer %d entry", i);
    if (int32_t rc = check_ternary(L.entry, name)) return rc;
    snprintf(name, sizeof(name), "layer %d out", i);
    if (int32_t rc = check_ternary(L.out, name)) return rc;
    snprintf(name, sizeof(name), "layer %d gate_up", i);
    if (int32_t rc = check_ternary(L.gate_up, name)) return rc;
    snprintf(name, sizeof(name), "layer %d down", i);
    if (int32_t rc = check_ternary(L.down, name)) return rc;
    if (L.entry.in_features != d.hidden || L.out.rows != d.hidden || L.gate_up.rows != 2 * d.dense ||
        L.down.rows != d.hidden || L.down.in_features != d.dense || L.gate_up.in_features != d.hidden ||
        L.out.in_features != d.hidden)
      return fail(IVB_EINVAL, "layer %d: projection shapes do not match the model dimensions", i);
    if (!L.mixer_norm || !L.ffn_norm) return fail(IVB_EINVAL, "layer %d: null norm weight", i);
    if (L.kind == IVB_MAMBA) {
      if (L.entry.rows != 2 * d.hidden + 3 * d.heads * d.state_dim)
        return fail(IVB_EINVAL, "layer %d: mamba entry must be [2*hidden + 3*heads*state, hidden]", i);
      if (!L.decay || !L.theta || !L.skip || !L.conv_weight || !L.conv_bias || !L.ssm_state || !L.prev_force ||
          !L.conv_state || L.conv_taps < 1)
        return fail(IVB_EINVAL, "layer %d: missing recurrent constants or state", i);
      if (taps >= 0 && taps != L.conv_taps) return fail(IVB_EINVAL, "all recurrent layers must share the conv width");
      taps = L.conv_taps;
    } else if (L.kind == IVB_MLA) {
      if (L.entry.rows != d.hidden + d.latent_dim + d.heads * d.rope_dim)
        return fail(IVB_EINVAL, "layer %d: mla entry must be [hidden + latent + heads*rope, hidden]", i);
      snprintf(name, sizeof(name), "layer %d k_nope_up", i);
      if (int32_t rc = check_ternary(L.k_nope_up, name)) return rc;
      snprintf(name, sizeof(name), "layer %d v_up", i);
      if (int32_t rc = check_ternary(L.v_up, name)) return rc;
      if (L.k_nope_up.rows != d.heads * d.nope_dim || L.k_nope_up.in_features != d.latent_dim ||
          L.v_up.rows != d.hidden || L.v_up.in_features != d.latent_dim)
        return fail(IVB_EINVAL, "layer %d: latent up-projections have the wrong shape", i);
      if (!L.rope || !L.latent_q || !L.latent_scale || !L.k_rope_cache)
        return fail(IVB_EINVAL, "layer %d: missing rope table or latent cache", i);
      if ((reinterpret_cast<uintptr_t>(L.latent_q) & 15) || (reinterpret_cast<uintptr_t>(L.latent_scale) & 15) ||
          (reinterpret_cast<uintptr_t>(L.k_rope_cache) & 15))
        return fail(IVB_EINVAL, "layer %d: the latent cache must be 16-byte aligned", i);
      if (!L.k_cache || !L.v_cache || (reinterpret_cast<uintptr_t>(L.k_cache) & 15) || (reinterpret_cast<uintptr_t>(L.v_cache) & 15))
        return fail(IVB_EINVAL, "layer %d: missing or unaligned key/value cache", i);
    } else {
      return fail(IVB_EINVAL, "layer %d: unknown kind %d", i, L.kind);
    }
  }
  return IVB_OK;
}

// True when every one of R CTAs gets at least one of n rows under the uniform partition ceil(n / R):
// then the gather of such an op waits for every CTA, which is what lets each op's flag-word buffer be
// reused every token (no CTA can be a whole token ahead of another one still reading it).
static bool every_cta_has_rows(int n, int R) {
  const int per = (n + R - 1) / R;
  return R <= n && per * (R - 1) < n;
}

// Builds the stream, op program, flag-word buffers and shared-memory map for R CTAs; false if it does not fit.
static bool plan(IvbDecoder* dec, int R, size_t smem_cap, std::string& why) {
  const IvbModelDesc& md = dec->desc;
  DecodeDims& D = dec->d;
  D = DecodeDims{};
  D.vocab = md.vocab;
  D.hidden = md.hidden;
  D.heads = md.heads;
  D.head_dim = md.head_dim;
  D.state_dim = md.state_dim;
  D.latent = md.latent_dim;
  D.rope = md.rope_dim;
  D.nope = md.nope_dim;
  D.dense = md.dense;
  D.max_len = md.max_len;
  D.max_top_k = md.max_top_k;
  D.R = R;
  D.taps = 1;
  D.act_eps = md.act_eps;
  D.clip = md.norm_clip;
  D.lpad = static_cast<int>(r16(md.latent_dim));
  D.kvpad = r4(md.head_dim);
  D.rpad = (md.rope_dim + 7) / 8 * 8;
  D.rb_lat = static_cast<int>(r16((md.latent_dim + 3) / 4));
  D.ss_lat = ((md.latent_dim + 127) / 128 + 7) / 8 * 8;
  for (const IvbLayerDesc& L : dec->layers) {
    if (L.kind == IVB_MAMBA) {
      D.taps = L.conv_taps;
      D.half_dt_min = L.half_dt_min;
      D.half_dt_range = L.half_dt_range;
    }
  }
  const int d = md.hidden, F = md.dense, Lt = md.latent_dim, hd = md.head_dim, S = md.state_dim, H = md.heads;
  // every GEMV CTA owns hidden / R recurrent channels inside one head and rows of every hidden/FFN projection
  if (d % R != 0 || R % H != 0 || !every_cta_has_rows(F, R)) {
    why = "the CTA count must divide the hidden width, be a multiple of the heads and leave every CTA FFN rows";
    return false;
  }
  if (d > kMaxEPT * kThreads || F > kMaxEPT * kThreads) {
    why = "hidden and FFN widths above 3072 are not supported by the decode kernel";
    return false;
  }
  D.cpc = d / R;
  // the recurrent state of a CTA's channels arrives by one 16-byte copy per thread when cpc is a power
  // of two of at least 4 and every piece is 16-byte aligned
  {
    int lg = 0;
    while ((2 << lg) < D.cpc) ++lg;  // cpc / 2 = 2^lg
    const int S = md.state_dim, taps = D.taps;
    const bool pow2 = D.cpc >= 4 && (2 << lg) == D.cpc;
    D.ssm_lg_cs = lg;
    D.ssm_v16 = pow2 && md.head_dim % 4 == 0 && (D.cpc * (taps - 1)) % 4 == 0 && ssm_state_off(D.cpc, S, taps) % 4 == 0 &&
                (S << lg) + (S << (lg - 1)) + (D.cpc * (taps - 1)) / 4 <= kThreads;
  }
  D.A = 0;
  for (const IvbLayerDesc& L : dec->layers)
    if (L.kind == IVB_MLA) D.A = H;
  const int cpc = D.cpc;
  const int dper = d / R, Fper = (F + R - 1) / R, Vper = (md.vocab + R - 1) / R;
  const int ent_mla = d + Lt + H * D.rope;  // rows of the mla entry matrix: [q | latent | k_rope]
  const int Eper = (ent_mla + R - 1) / R;
  auto part = [&](int n, int per, int c) { return std::max(0, std::min(n, (c + 1) * per) - std::min(n, c * per)); };
  const size_t stage = 20 * 1024;
  dec->kc = std::min(std::min(md.max_top_k, md.vocab), kMaxTopK);
  if (Vper > kThreads) {
    why = "more than 256 vocabulary rows per CTA";
    return false;
  }
  // ---- op program and per-CTA segments ------------------------------------------------------------
  struct OpPlan {
    Op op;
    std::vector<std::vector<Segment>> segs;  // [R] row segments of each CTA
    int const_kind;                           // 0 none, 2 mamba (ssm constants), 3 attention
    const float* norm;
    const IvbLayerDesc* layer;
    int out_words;                            // flag words of the op's output vector
  };
  std::vector<OpPlan> plans;
  auto gemv_op = [&](int kind, int layer, const IvbTernary& m, int in_n, int rows_per, int rows_total, int in_dst,
                     const float* norm, float eps) {
    OpPlan pl{};
    pl.op.kind = kind;
    pl.op.layer = layer;
    pl.op.in_dst = in_dst;
    pl.op.in_n = in_n;
    pl.op.rows_per = rows_per;
    pl.op.rows_total = rows_total;
    // the chunk's row stride: the packed row, plus 16 bytes when it is a multiple of 128 bytes, so the
    // rows of one warp's 16-byte weight loads fall on different shared-memory banks
    pl.op.row_bytes = m.row_bytes % 128 == 0 ? m.row_bytes + 16 : m.row_bytes;
    pl.op.scale_stride = ((m.in_features + 127) / 128 + 7) / 8 * 8;
    pl.op.has_bias = m.bias != nullptr;
    // lanes per row: at most kRowsKPL chunks per lane, then as many lanes as keep the CTA's rows in one
    // pass of rows_generic (rows x lanes <= 256) without idle lanes (lanes <= chunks), at most 16 (the
    // lane butterfly stays at four steps, and gate/up row pairs share a warp)
    const int chunks = (in_n + 63) / 64;
    int lg = 0;
    while (lg < 5 && ((chunks + (1 << lg) - 1) >> lg) > kRowsKPL) ++lg;
    while (lg < 4 && (1 << (lg + 1)) <= chunks && (std::max(rows_per, 1) << (lg + 1)) <= kThreads) ++lg;
    pl.op.lpr_log = lg;
    pl.op.has_norm = norm != nullptr;
    pl.op.has_norm_chunk = norm != nullptr;
    pl.op.norm_eps = eps;
    pl.norm = norm;
    pl.const_kind = 0;
    pl.segs.assign(R, {});
    return pl;
  };
  for (int li = 0; li < static_cast<int>(dec->layers.size()); ++li) {
    const IvbLayerDesc& L = dec->layers[li];
    if (L.kind == IVB_MAMBA) {
      // value and gate rows of my channels, then the B, C, dt rows of their head
      OpPlan e = gemv_op(OP_ENTRY_MAMBA, li, L.entry, d, 2 * cpc + 3 * S, R * (2 * cpc + 3 * S), IN_RESID, L.mixer_norm,
                         L.mixer_norm_eps);
      e.const_kind = 2;
      e.layer = &L;
      e.out_words = d;
      for (int c = 0; c < R; ++c) {
        const int ch0 = c * cpc, h = ch0 / hd;
        e.segs[c].push_back({&L.entry, ch0, cpc});
        e.segs[c].push_back({&L.entry, d + ch0, cpc});
        e.segs[c].push_back({&L.entry, 2 * d + h * 3 * S, 3 * S});
      }
      plans.push_back(e);
    } else {
      OpPlan e = gemv_op(OP_ENTRY_MLA, li, L.entry, d, Eper, ent_mla, IN_RESID, L.mixer_norm, L.mixer_norm_eps);
      e.layer = &L;
      e.out_words = ent_mla;
      for (int c = 0; c < R; ++c)
        if (part(ent_mla, Eper, c) > 0) e.segs[c].push_back({&L.entry, c * Eper, part(ent_mla, Eper, c)});
      plans.push_back(e);
      OpPlan a{};
      a.op.kind = OP_ATTN;
      a.op.layer = li;
      a.op.in_dst = IN_LATENT;
      a.op.in_n = Lt;
      // the head's kv up-projection rows (k_nope, then v) as one GEMV row chunk of its stream
      a.op.rows_per = D.nope + hd;
      a.op.rows_total = 0;
      a.op.row_bytes = D.rb_lat;
      a.op.scale_stride = D.ss_lat;
      a.op.has_bias = 1;
      {
        const int chunks = (Lt + 63) / 64;
        int lg = 0;
        while (lg < 5 && ((chunks + (1 << lg) - 1) >> lg) > kRowsKPL) ++lg;
        while (lg < 4 && (1 << (lg + 1)) <= chunks && (a.op.rows_per << (lg + 1)) <= kThreads) ++lg;
        a.op.lpr_log = lg;
      }
      a.const_kind = 3;
      a.layer = &L;
      a.out_words = d;  // the heads' outputs, written by the attention CTAs
      a.segs.assign(R, {});
      plans.push_back(a);
    }
    OpPlan o = gemv_op(OP_OUT, li, L.out, d, dper, d, IN_VEC, nullptr, 0.0f);
    o.out_words = d;
    for (int c = 0; c < R; ++c) o.segs[c].push_back({&L.out, c * dper, dper});
    plans.push_back(o);
    OpPlan g = gemv_op(OP_GATE_UP, li, L.gate_up, d, 2 * Fper, 2 * F, IN_RESID, L.ffn_norm, L.ffn_norm_eps);
    g.out_words = F;
    for (int c = 0; c < R; ++c)
      if (part(F, Fper, c) > 0) g.segs[c].push_back({&L.gate_up, 2 * c * Fper, 2 * part(F, Fper, c)});
    plans.push_back(g);
    OpPlan dn = gemv_op(OP_DOWN, li, L.down, F, dper, d, IN_VEC, nullptr, 0.0f);
    dn.out_words = d;
    for (int c = 0; c < R; ++c) dn.segs[c].push_back({&L.down, c * dper, dper});
    plans.push_back(dn);
  }
  const int kp_max = (std::min(dec->kc, std::max(Vper, 1)) + 1) & ~1;  // candidate slots per CTA (cand_slots)
  {
    OpPlan hp = gemv_op(OP_HEAD, -1, md.head, d, Vper, md.vocab, IN_RESID, md.final_norm, md.final_norm_eps);
    hp.out_words = 2 * R * kp_max;
    for (int c = 0; c < R; ++c)
      if (part(md.vocab, Vper, c) > 0) hp.segs[c].push_back({&md.head, c * Vper, part(md.vocab, Vper, c)});
    plans.push_back(hp);
    OpPlan mg{};
    mg.op.kind = OP_MERGE;
    mg.op.layer = -1;
    mg.op.in_dst = IN_CAND;
    mg.const_kind = 0;
    mg.out_words = 0;  // set with the group size below
    mg.segs.assign(R, {});
    plans.push_back(mg);
  }
  // ---- constants-chunk layouts (identical offsets for every CTA) ----------------------------------
  // The norm weights are their own chunk, read in place from the model's array when it is 16-byte
  // aligned (one shared copy for all CTAs instead of one per CTA); the per-CTA constants of the
  // recurrent step (its head's decay/theta, its channels' skip and conv) and of the attention (its
  // head's up-projection rows) live in a constants chunk of the stream.
  const bool norm_in_place = (d * 4) % 16 == 0;
  size_t max_const = 16;
  for (OpPlan& pl : plans) {
    Op& op = pl.op;
    size_t off = 0;
    if (pl.const_kind == 2) {
      op.c_decay = static_cast<int>(off);
      off += r16(S * 4);
      op.c_theta = static_cast<int>(off);
      off += r16(S * 4);
      op.c_skip = static_cast<int>(off);
      off += r16(cpc * 4);
      op.c_convw = static_cast<int>(off);
      off += r16(static_cast<size_t>(cpc) * D.taps * 4);
      op.c_convb = static_cast<int>(off);
      off += r16(cpc * 4);
    }
    if (pl.const_kind == 3) {  // [k x row_bytes][k x scale_stride fp16, 16B pad][k x fp32 bias], k = nope + hd
      const size_t k = static_cast<size_t>(D.nope + hd);
      off = k * D.rb_lat + r16(k * D.ss_lat * 2) + r16(k * 4);
    }
    op.has_const = pl.const_kind != 0;
    max_const = std::max(max_const, off);
    if (op.has_norm_chunk) max_const = std::max(max_const, r16(static_cast<size_t>(d) * 4));
    pl.op.n_chunks = 0;
  }
  if (max_const > stage) {
    why = "a constants chunk does not fit a stream stage";
    return false;
  }
  // ---- chunk the rows ---------------------------------------------------------------------------
  for (OpPlan& pl : plans) {
    Op& op = pl.op;
    if (op.kind == OP_ATTN) {  // its constants chunk is in the attention CTAs' own streams
      op.chunk_rows = 0;
      op.n_chunks = 0;
      op.has_const = 0;
      continue;
    }
    if (op.kind == OP_MERGE) {
      op.chunk_rows = 0;
      op.n_chunks = 0;
      continue;
    }
    const size_t per_row = op.row_bytes + op.scale_stride * 2 + 4;
    int cr = static_cast<int>((stage - 64) / per_row);
    const int rpi = kThreads >> op.lpr_log;  // rows one pass of rows_generic covers
    if (cr >= rpi) cr = cr / rpi * rpi;
    if (op.kind == OP_GATE_UP) cr &= ~1;
    cr = std::max(2, std::min(cr, std::max(2, op.rows_per)));
    op.chunk_rows = cr;
    op.n_chunks = op.has_norm_chunk + op.has_const + (op.rows_per + cr - 1) / cr;
  }
  // ---- shared memory map ----------------------------------------------------------------------------
  // [fixed regions][union region][ring of kStages stages]: a GEMV CTA's union region ends where the ring
  // starts; an attention CTA streams through the ring's last kAttnStages stages only, so its union region
  // (the attention tiles) runs on through the others
  DecodeSmem& M = dec->sm;
  size_t o = 0;
  M.stage_bytes = static_cast<int>(stage);
  const size_t ring_bytes = kStages * stage, attn_ring_bytes = kAttnStages * stage;
  const int max_in = std::max(std::max(d, F), Lt);  // GEMV inputs, the latent's codes included
  const int pad_in = (max_in + 63) / 64 * 64;
  M.act = static_cast<int>(o);
  o += r16(pad_in);
  M.xsum = static_cast<int>(o);
  o += r16(pad_in / 64 * 8);  // two half-chunk code sums per 64-input chunk
  M.resid = static_cast<int>(o);
  o += r16(static_cast<size_t>(d) * 4);
  int pub_n = std::max(std::max(cpc, hd + 2), std::max(dper, Fper));
  M.pub_n = pub_n;
  M.pub = static_cast<int>(o);
  o += r16(static_cast<size_t>(pub_n) * 4);  // staging of the op's output slice
  int loc_n = 0;
  for (const OpPlan& pl : plans) loc_n = std::max(loc_n, pl.op.rows_per);
  M.loc = static_cast<int>(o);
  o += r16(static_cast<size_t>(loc_n) * 4);
  M.red = static_cast<int>(o);
  o += r16(64 * 4);
  M.xl = static_cast<int>(o);
  o += r16(static_cast<size_t>((hd + Lt + D.rope + 63) / 64 * 64) * 4);
  int cpt = 0;
  for (const OpPlan& pl : plans) cpt += pl.op.n_chunks;
  M.ctab = static_cast<int>(o);
  o += r16(static_cast<size_t>(cpt) * 8) + r16(static_cast<size_t>(cpt) * 4);
  M.rope_row = static_cast<int>(o);
  o += r16(static_cast<size_t>(std::max(md.rope_dim, 1)) * 4);
  M.seen = static_cast<int>(o);
  o += r16(static_cast<size_t>(Vper));
  M.u = static_cast<int>(o);
  if (o + ring_bytes >= smem_cap) {
    why = "the decoder's fixed shared-memory regions exceed a CTA's shared memory";
    return false;
  }
  const int kc = dec->kc;
  const size_t room = smem_cap - o - ring_bytes;  // a GEMV CTA's union region
  // recurrent op: constants, scratch and prefetched state of the CTA's channels
  size_t u_need = r16(static_cast<size_t>(ssm_smem_floats(cpc, S, D.taps)) * 4);
  // head: keys [256] and its candidates [kc]; merges: scratch, then the gathered candidate arrays
  const size_t head_scratch = static_cast<size_t>(kThreads) * 4 + 2 * static_cast<size_t>(kc) * 4;
  const size_t merge_scratch = 5 * static_cast<size_t>(kc) * 4 + kWarps * 256 * 4 + 16 * 4;
  M.cand = static_cast<int>(r16(std::max(head_scratch, merge_scratch)));
  if (static_cast<size_t>(M.cand) + 16 * 8 > room) {
    why = "no room for the sampler's candidates in shared memory";
    return false;
  }
  // candidates one merge can hold: all of them when they fit, else groups of CTAs whose leaders merge first
  const size_t cap_c = std::min<size_t>((room - M.cand) / 8, static_cast<size_t>(R) * kp_max);
  D.cand_cap = static_cast<int>(cap_c);
  D.group = R;
  if (static_cast<size_t>(R) * kp_max > cap_c) {
    int g = static_cast<int>(cap_c / kp_max);
    for (; g >= 1; --g) {
      const int ng = (R + g - 1) / g;
      const int kq = (std::min(kc, g * kp_max) + 1) & ~1;
      if (static_cast<size_t>(ng) * kq <= cap_c) break;
    }
    if (g < 1) {
      why = "the sampler's candidate merge does not fit shared memory";
      return false;
    }
    D.group = g;
  }
  {
    const int ng = (R + D.group - 1) / D.group;
    const int kq = (std::min(kc, D.group * kp_max) + 1) & ~1;
    plans.back().out_words = 2 * ng * kq;
  }
  u_need = std::max(u_need, static_cast<size_t>(M.cand) + r16(cap_c * 8));
  bool any_mla = false;
  for (const IvbLayerDesc& L : dec->layers) any_mla |= L.kind == IVB_MLA;
  int tile = 0;
  if (any_mla) {
    // two tile buffers of tile + 1 rows (the last tile also holds the current position)
    auto attn_bytes = [&](int t) { return attn_fixed_bytes(D.nope, hd) + 4 * tile_bytes(t, D.kvpad); };
    const size_t attn_room = smem_cap - o - attn_ring_bytes;
    // at most 240 positions: a tile and the current row then take at most 8 passes of 32 (attn_tiles)
    tile = std::min(240, (md.max_len + 15) / 16 * 16);
    while (tile >= 16 && attn_bytes(tile) > attn_room) tile -= 16;
    if (tile < 16) {
      why = "no room for an attention tile in shared memory";
      return false;
    }
    // the ring starts late enough for the attention region to end at its last kAttnStages stages
    const size_t attn_end = o + r16(attn_bytes(tile));
    const size_t ring_lo = attn_end > (ring_bytes - attn_ring_bytes) ? attn_end - (ring_bytes - attn_ring_bytes) : 0;
    u_need = std::max(u_need, r16(ring_lo > o ? ring_lo - o : 0));
  }
  D.tile = std::max(tile, 16);
  o += r16(u_need);
  M.ring = static_cast<int>(o);
  o += ring_bytes;
  M.total = static_cast<int>(o);
  if (o > smem_cap) {
    why = "the decoder needs more shared memory than a CTA has";
    return false;
  }
  dec->smem = o;
  // ---- op records: chunks, flag-word buffers ---------------------------------------------------------
  dec->ops.clear();
  dec->op_rows.assign(plans.size() * R, 0);
  cpt = 0;
  size_t llw = 0;
  for (size_t i = 0; i < plans.size(); ++i) {
    Op& op = plans[i].op;
    op.first_chunk = cpt;
    cpt += op.n_chunks;
    op.ll_out = static_cast<int32_t>(llw);
    llw += (static_cast<size_t>(plans[i].out_words) + 15) / 16 * 16;  // whole 128-byte lines per buffer
    const bool first_entry = (op.kind == OP_ENTRY_MAMBA || op.kind == OP_ENTRY_MLA) && op.layer == 0;
    if (i == 0 || first_entry) {
      op.ll_in = -1;
      op.ll_in_words = 0;
    } else {
      op.ll_in = plans[i - 1].op.ll_out;
      op.ll_in_words = plans[i - 1].out_words;
    }
    if (op.kind == OP_HEAD) dec->head_op = static_cast<int32_t>(i);
    dec->ops.push_back(op);
  }
  dec->ll_words = llw;
  dec->cpt = cpt;
  dec->head_first = plans[dec->head_op].op.first_chunk;
  // ---- every CTA's stream ---------------------------------------------------------------------------
  dec->chunk_off.assign(static_cast<size_t>(R) * cpt, 0);
  dec->chunk_ptr.assign(static_cast<size_t>(R) * cpt, 0);
  dec->chunk_bytes.assign(static_cast<size_t>(R) * cpt, 0);
  dec->copies.clear();
  size_t cursor = 0;
  auto add = [&](size_t dst, const void* src, size_t width, size_t rows, size_t spitch, size_t dpitch) {
    if (width == 0 || rows == 0) return;
    dec->copies.push_back(CopyOp{dst, src, width, rows, spitch, dpitch});
  };
  for (int c = 0; c < R; ++c) {
    int ci = 0;
    for (size_t i = 0; i < plans.size(); ++i) {
      const OpPlan& pl = plans[i];
      const Op& op = pl.op;
      int rows_c = 0;
      for (const Segment& sg : pl.segs[c]) rows_c += sg.count;
      dec->op_rows[i * R + c] = rows_c;
      if (op.has_norm_chunk) {
        const size_t nb = r16(static_cast<size_t>(d) * 4);
        if (norm_in_place && (reinterpret_cast<uintptr_t>(pl.norm) & 15) == 0) {
          dec->chunk_off[static_cast<size_t>(c) * cpt + ci] = ~0ull;
          dec->chunk_ptr[static_cast<size_t>(c) * cpt + ci] = reinterpret_cast<uintptr_t>(pl.norm);
        } else {
          add(cursor, pl.norm, static_cast<size_t>(d) * 4, 1, 0, 0);
          dec->chunk_off[static_cast<size_t>(c) * cpt + ci] = cursor;
          cursor = r16(cursor + nb);
        }
        dec->chunk_bytes[static_cast<size_t>(c) * cpt + ci] = static_cast<unsigned>(nb);
        ++ci;
      }
      if (op.has_const) {
        const size_t base = cursor;
        size_t bytes = 16;
        if (pl.const_kind == 2) {
          const IvbLayerDesc& L = *pl.layer;
          const int ch0 = c * cpc, h = ch0 / hd;
          add(base + op.c_decay, L.decay + h * S, S * 4, 1, 0, 0);
          add(base + op.c_theta, L.theta + h * S, S * 4, 1, 0, 0);
          add(base + op.c_skip, L.skip + ch0, cpc * 4, 1, 0, 0);
          add(base + op.c_convw, L.conv_weight + static_cast<size_t>(ch0) * D.taps, static_cast<size_t>(cpc) * D.taps * 4, 1, 0, 0);
          add(base + op.c_convb, L.conv_bias + ch0, cpc * 4, 1, 0, 0);
          bytes = std::max(bytes, static_cast<size_t>(op.c_convb) + r16(cpc * 4));
        }
        dec->chunk_off[static_cast<size_t>(c) * cpt + ci] = base;
        dec->chunk_bytes[static_cast<size_t>(c) * cpt + ci] = static_cast<unsigned>(r16(bytes));
        cursor = r16(base + bytes);
        ++ci;
      }
      if (op.kind == OP_ATTN || op.kind == OP_MERGE) continue;
      // row chunks: [k x row_bytes][k x scale_stride fp16, 16B pad][k x fp32 bias, 16B pad]
      const int n_row_chunks = op.n_chunks - op.has_const - op.has_norm_chunk;
      for (int rc = 0; rc < n_row_chunks; ++rc) {
        const int r0 = rc * op.chunk_rows;
        const int k = std::max(0, std::min(op.chunk_rows, rows_c - r0));
        const size_t base = cursor;
        const size_t sc_off = static_cast<size_t>(k) * op.row_bytes;
        const size_t b_off = sc_off + r16(static_cast<size_t>(k) * op.scale_stride * 2);
        const size_t bytes = std::max<size_t>(16, b_off + r16(static_cast<size_t>(k) * 4));
        // walk the segments covering virtual rows [r0, r0 + k)
        int v = 0;
        for (const Segment& sg : pl.segs[c]) {
          const int a = std::max(r0, v), b = std::min(r0 + k, v + sg.count);
          if (a < b) {
            const int src_row = sg.row0 + (a - v);
            const int n = b - a;
            const IvbTernary& m = *sg.m;
            const size_t dr = static_cast<size_t>(a - r0);
            add(base + dr * op.row_bytes, m.packed + static_cast<size_t>(src_row) * m.row_bytes, m.row_bytes, n, m.row_bytes,
                op.row_bytes);
            add(base + sc_off + dr * op.scale_stride * 2, m.scales + static_cast<size_t>(src_row) * m.scale_stride,
                static_cast<size_t>((m.in_features + 127) / 128) * 2, n, static_cast<size_t>(m.scale_stride) * 2,
                static_cast<size_t>(op.scale_stride) * 2);
            if (op.has_bias) add(base + b_off + dr * 4, m.bias + src_row, static_cast<size_t>(n) * 4, 1, 0, 0);
          }
          v += sg.count;
        }
        dec->chunk_off[static_cast<size_t>(c) * cpt + ci] = base;
        dec->chunk_bytes[static_cast<size_t>(c) * cpt + ci] = static_cast<unsigned>(r16(bytes));
        cursor = r16(base + bytes);
        ++ci;
      }
    }
  }
  // the attention CTAs' streams: per head, one constants chunk per attention op (the head's k_nope and
  // v up-projection rows, scales and biases)
  dec->attn_ops.clear();
  for (size_t i = 0; i < plans.size(); ++i)
    if (plans[i].op.kind == OP_ATTN) dec->attn_ops.push_back(static_cast<int32_t>(i));
  const int n_mla = static_cast<int>(dec->attn_ops.size());
  dec->A = n_mla > 0 ? H : 0;
  dec->attn_off.assign(static_cast<size_t>(dec->A) * n_mla, 0);
  dec->attn_bytes.assign(static_cast<size_t>(dec->A) * n_mla, 16);
  for (int h = 0; h < dec->A; ++h)
    for (int mi = 0; mi < n_mla; ++mi) {
      const OpPlan& pl = plans[dec->attn_ops[mi]];
      const IvbLayerDesc& L = *pl.layer;
      const IvbTernary& kn = L.k_nope_up;
      const IvbTernary& vu = L.v_up;
      const size_t sgroups = static_cast<size_t>((Lt + 127) / 128) * 2;
      const size_t base = cursor, k = static_cast<size_t>(D.nope + hd), nn = static_cast<size_t>(D.nope);
      const size_t sc_off = k * D.rb_lat, b_off = sc_off + r16(k * D.ss_lat * 2);
      // rows [0, nope): k_nope rows of head h; rows [nope, nope + hd): its v rows (absent biases are zero)
      add(base, kn.packed + static_cast<size_t>(h) * D.nope * kn.row_bytes, D.rb_lat, nn, kn.row_bytes, D.rb_lat);
      add(base + nn * D.rb_lat, vu.packed + static_cast<size_t>(h) * hd * vu.row_bytes, D.rb_lat, hd, vu.row_bytes, D.rb_lat);
      add(base + sc_off, kn.scales + static_cast<size_t>(h) * D.nope * kn.scale_stride, sgroups, nn,
          static_cast<size_t>(kn.scale_stride) * 2, static_cast<size_t>(D.ss_lat) * 2);
      add(base + sc_off + nn * D.ss_lat * 2, vu.scales + static_cast<size_t>(h) * hd * vu.scale_stride, sgroups, hd,
          static_cast<size_t>(vu.scale_stride) * 2, static_cast<size_t>(D.ss_lat) * 2);
      add(base + b_off, kn.bias ? static_cast<const void*>(kn.bias + h * D.nope) : nullptr, nn * 4, 1, 0, 0);
      add(base + b_off + nn * 4, vu.bias ? static_cast<const void*>(vu.bias + h * hd) : nullptr, static_cast<size_t>(hd) * 4, 1, 0, 0);
      const size_t bytes = r16(b_off + r16(k * 4));
      dec->attn_off[static_cast<size_t>(h) * n_mla + mi] = base;
      dec->attn_bytes[static_cast<size_t>(h) * n_mla + mi] = static_cast<unsigned>(bytes);
      cursor = r16(base + bytes);
    }
  dec->stream_bytes = r16(cursor) + 256;
  // ---- consistency of the plan (checked here so that a planning error is an error code, not a fault) --
  for (size_t i = 0; i < dec->attn_bytes.size(); ++i)
    if (dec->attn_bytes[i] > stage || dec->attn_off[i] + dec->attn_bytes[i] > dec->stream_bytes) {
      why = "an attention constants chunk does not fit a ring stage";
      return false;
    }
  for (size_t i = 0; i < dec->chunk_bytes.size(); ++i) {
    const unsigned b = dec->chunk_bytes[i];
    if (b == 0 || b > stage || (b & 15) != 0) {
      why = "a stream chunk does not fit a ring stage";
      return false;
    }
    if (dec->chunk_off[i] != ~0ull && dec->chunk_off[i] + b > dec->stream_bytes) {
      why = "a stream chunk lies outside the stream";
      return false;
    }
  }
  for (size_t i = 0; i < plans.size(); ++i) {
    const Op& op = dec->ops[i];
    if (op.n_chunks > kStages) {
      why = "an op needs more stream chunks than the ring holds";
      return false;
    }
    if (static_cast<size_t>(op.ll_out) + plans[i].out_words > dec->ll_words) {
      why = "a flag-word buffer lies outside its region";
      return false;
    }
    for (int c = 0; c < R; ++c) {
      const int rows_c = dec->op_rows[i * R + c];
      if (op.kind != OP_ATTN && op.kind != OP_MERGE && (rows_c > op.rows_per || rows_c > loc_n)) {
        why = "a CTA's rows exceed its row buffer";
        return false;
      }
    }
  }
  return true;
}

}  // namespace ivb

namespace ivb {
// The model description and layers a decoder was created with (for the prefill path).
const IvbModelDesc& decoder_model(const IvbDecoder* dec, const IvbLayerDesc** layers) {
  *layers = dec->layers.data();
  return dec->desc;
}
// The device error word ivb_decoder_check reports (nullptr before bind).
unsigned* decoder_error_word(const IvbDecoder* dec) {
  return dec->ws == nullptr ? nullptr : reinterpret_cast<unsigned*>(dec->ws + dec->off_sync);
}
}  // namespace ivb

extern "C" {

int32_t ivb_decode_rows(const uint8_t* stage, int32_t k, int32_t row_bytes, int32_t scale_stride, int32_t has_bias,
                        float act_scale, const int8_t* q8, int32_t in_n, int32_t lanes_log, float* out, void* stream) {
  using namespace ivb;
  if (stage == nullptr || q8 == nullptr || out == nullptr) return fail(IVB_EINVAL, "ivb_decode_rows: null argument");
  if (k <= 0 || in_n <= 0 || lanes_log < -1 || lanes_log > 5 || scale_stride <= 0)
    return fail(IVB_EINVAL, "ivb_decode_rows: bad shape");
  if ((row_bytes & 15) != 0 || row_bytes < (in_n + 3) / 4)
    return fail(IVB_EINVAL, "ivb_decode_rows: row_bytes must be a multiple of 16 holding the row");
  const int chunks = (in_n + 63) / 64;
  if (chunks > (kRowsKPL << (lanes_log < 0 ? 4 : lanes_log)))
    return fail(IVB_EINVAL, "ivb_decode_rows: more than %d chunks per lane", kRowsKPL);
  const size_t stage_bytes = static_cast<size_t>(k) * row_bytes + round16(static_cast<size_t>(k) * scale_stride * 2) +
                             (has_bias ? static_cast<size_t>(k) * 4 : 0);
  const size_t smem = round16(stage_bytes) + static_cast<size_t>(chunks) * 64 + static_cast<size_t>(chunks) * 8 + static_cast<size_t>(k) * 4;
  if (smem > 200 * 1024) return fail(IVB_EINVAL, "ivb_decode_rows: the chunk does not fit shared memory");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  IVB_CUDA(cudaFuncSetAttribute(rows_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  rows_probe_kernel<<<1, kThreads, smem, s>>>(stage, static_cast<int>(stage_bytes), k, row_bytes, scale_stride, has_bias,
                                              act_scale, q8, in_n, lanes_log, out);
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

int32_t ivb_decoder_create(const IvbModelDesc* desc, int32_t ctas, IvbDecoder** out) {
  using namespace ivb;
  if (desc == nullptr || out == nullptr) return fail(IVB_EINVAL, "ivb_decoder_create: null argument");
  *out = nullptr;
  if (int32_t rc = validate(*desc)) return rc;
  IvbDecoder* dec = new (std::nothrow) IvbDecoder();
  if (dec == nullptr) return fail(IVB_EINVAL, "out of host memory");
  dec->desc = *desc;
  dec->layers.assign(desc->layers, desc->layers + desc->num_layers);
  dec->desc.layers = nullptr;
  dec->ws = nullptr;
  dec->trace = nullptr;
  dec->trace_step = 0;
  int dev = 0, optin = 0, sms = 0;
  IVB_CUDA(cudaGetDevice(&dev));
  IVB_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  IVB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const size_t cap = static_cast<size_t>(optin) - 4096;  // static shared memory of the kernel
  // CTA count: the request (default 128: the flag-word handoff measured fastest there on B200), at
  // most one CTA per SM, lowered until every CTA has rows of every hidden/FFN projection and the
  // plan fits a CTA's shared memory
  const int want = std::min(ctas > 0 ? ctas : 128, sms - desc->heads);  // the attention CTAs take one SM per head
  std::string why = "no CTA count fits";
  bool planned = false;
  for (int R = want; R >= 1; --R) {
    std::string w;
    if (!plan(dec, R, cap, w)) {
      if (why == "no CTA count fits") why = w;
      continue;
    }
    IVB_CUDA(cudaFuncSetAttribute(grid_decode_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dec->smem)));
    IVB_CUDA(cudaFuncSetAttribute(grid_decode_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dec->smem)));
    int per_sm = 0, per_sm_trace = 0;
    IVB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, grid_decode_kernel<false>, kThreads, dec->smem));
    IVB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_trace, grid_decode_kernel<true>, kThreads, dec->smem));
    per_sm = std::min(per_sm, per_sm_trace);
    if (per_sm < 1 || per_sm * sms < R + dec->A) {
      why = "the device cannot hold every CTA of the decode kernel at once";
      continue;
    }
    dec->R = R;
    planned = true;
    break;
  }
  if (!planned) {
    delete dec;
    return fail(IVB_EINVAL, "ivb_decoder_create: %s", why.c_str());
  }
  size_t off = 0;
  dec->off_stream = off;
  off = align_up(off + dec->stream_bytes, 256);
  dec->off_ops = off;
  off = align_up(off + dec->ops.size() * sizeof(OpRec), 256);
  dec->off_op_rows = off;
  off = align_up(off + dec->op_rows.size() * 4, 256);
  dec->off_chunk_addr = off;
  off = align_up(off + dec->chunk_off.size() * 8, 256);
  dec->off_chunk_bytes = off;
  off = align_up(off + dec->chunk_bytes.size() * 4, 256);
  dec->off_attn_addr = off;
  off = align_up(off + dec->attn_off.size() * 8 + 8, 256);
  dec->off_attn_bytes = off;
  off = align_up(off + dec->attn_bytes.size() * 4 + 4, 256);
  dec->off_attn_ops = off;
  off = align_up(off + dec->attn_ops.size() * 4 + 4, 256);
  dec->off_ll = off;
  off = align_up(off + dec->ll_words * 8, 256);
  dec->off_sync = off;  // [0] error word, [4] token epoch
  off = align_up(off + 256, 256);
  dec->total = off;
  *out = dec;
  return IVB_OK;
}

void ivb_decoder_destroy(IvbDecoder* dec) { delete dec; }

uint64_t ivb_decoder_workspace_bytes(const IvbDecoder* dec) { return dec ? dec->total : 0; }

int32_t ivb_decoder_num_phases(const IvbDecoder* dec) { return dec ? static_cast<int32_t>(dec->ops.size()) : 0; }

int32_t ivb_decoder_ctas(const IvbDecoder* dec) { return dec ? dec->R + dec->A : 0; }

int32_t ivb_decoder_bind(IvbDecoder* dec, void* workspace, void* stream) {
  using namespace ivb;
  if (dec == nullptr || workspace == nullptr) return fail(IVB_EINVAL, "ivb_decoder_bind: null argument");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return fail(IVB_EINVAL, "workspace must be 256-byte aligned");
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  dec->ws = ws;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned char* blob = ws + dec->off_stream;
  IVB_CUDA(cudaMemsetAsync(blob, 0, dec->stream_bytes, s));
  for (const CopyOp& c : dec->copies) {
    if (c.src == nullptr) {
      IVB_CUDA(cudaMemsetAsync(blob + c.dst, 0, c.width * c.rows, s));
    } else if (c.rows == 1) {
      IVB_CUDA(cudaMemcpyAsync(blob + c.dst, c.src, c.width, cudaMemcpyDeviceToDevice, s));
    } else {
      IVB_CUDA(cudaMemcpy2DAsync(blob + c.dst, c.dpitch, c.src, c.spitch, c.width, c.rows, cudaMemcpyDeviceToDevice, s));
    }
  }
  {
    dec->recs.assign(dec->ops.size(), OpRec{});
    for (size_t i = 0; i < dec->ops.size(); ++i) {
      std::memset(&dec->recs[i], 0, sizeof(OpRec));
      dec->recs[i].op = dec->ops[i];
      if (dec->ops[i].layer >= 0) dec->recs[i].layer = dec->layers[dec->ops[i].layer];
    }
    IVB_CUDA(cudaMemcpyAsync(ws + dec->off_ops, dec->recs.data(), dec->recs.size() * sizeof(OpRec), cudaMemcpyHostToDevice, s));
  }
  dec->chunk_addr.resize(dec->chunk_off.size());
  for (size_t i = 0; i < dec->chunk_off.size(); ++i)
    dec->chunk_addr[i] = dec->chunk_off[i] == ~0ull ? dec->chunk_ptr[i]
                                                    : static_cast<unsigned long long>(reinterpret_cast<uintptr_t>(blob)) + dec->chunk_off[i];
  IVB_CUDA(cudaMemcpyAsync(ws + dec->off_op_rows, dec->op_rows.data(), dec->op_rows.size() * 4, cudaMemcpyHostToDevice, s));
  IVB_CUDA(cudaMemcpyAsync(ws + dec->off_chunk_addr, dec->chunk_addr.data(), dec->chunk_addr.size() * 8, cudaMemcpyHostToDevice, s));
  IVB_CUDA(cudaMemcpyAsync(ws + dec->off_chunk_bytes, dec->chunk_bytes.data(), dec->chunk_bytes.size() * 4, cudaMemcpyHostToDevice, s));
  dec->attn_addr.resize(dec->attn_off.size());
  for (size_t i = 0; i < dec->attn_off.size(); ++i)
    dec->attn_addr[i] = static_cast<unsigned long long>(reinterpret_cast<uintptr_t>(blob)) + dec->attn_off[i];
  if (!dec->attn_addr.empty()) {
    IVB_CUDA(cudaMemcpyAsync(ws + dec->off_attn_addr, dec->attn_addr.data(), dec->attn_addr.size() * 8, cudaMemcpyHostToDevice, s));
    IVB_CUDA(cudaMemcpyAsync(ws + dec->off_attn_bytes, dec->attn_bytes.data(), dec->attn_bytes.size() * 4, cudaMemcpyHostToDevice, s));
    IVB_CUDA(cudaMemcpyAsync(ws + dec->off_attn_ops, dec->attn_ops.data(), dec->attn_ops.size() * 4, cudaMemcpyHostToDevice, s));
  }
  IVB_CUDA(cudaMemsetAsync(ws + dec->off_ll, 0, dec->ll_words * 8, s));  // every flag word starts at epoch 0
  IVB_CUDA(cudaMemsetAsync(ws + dec->off_sync, 0, 256, s));
  IVB_CUDA(cudaStreamSynchronize(s));
  return IVB_OK;
}

int32_t ivb_decoder_run(IvbDecoder* dec, int32_t steps, const int64_t* feed, int32_t flags, uint64_t timeout_ns,
                        void* stream) {
  using namespace ivb;
  if (dec == nullptr || dec->ws == nullptr) return fail(IVB_EINVAL, "ivb_decoder_run: decoder not bound");
  if (steps < 0) return fail(IVB_EINVAL, "ivb_decoder_run: negative step count");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned char* ws = dec->ws;
  unsigned* error = reinterpret_cast<unsigned*>(ws + dec->off_sync);
  const IvbModelDesc& md = dec->desc;
  if (flags & IVB_RUN_SAMPLE_ONLY) {
    IVB_CUDA(cudaMemsetAsync(error, 0, 4, s));
    return ivb_sample(md.logits, md.seen, md.vocab, md.sampling, md.top_k, md.max_top_k, md.rng, md.token, nullptr, stream);
  }
  if (steps == 0) return IVB_OK;
  if (feed == nullptr && !(flags & IVB_RUN_SAMPLE))
    return fail(IVB_EINVAL, "ivb_decoder_run: without fed tokens every step must sample");
  DecodeParams p{};
  p.ops = reinterpret_cast<const OpRec*>(ws + dec->off_ops);
  p.op_rows = reinterpret_cast<const int32_t*>(ws + dec->off_op_rows);
  p.n_ops = static_cast<int32_t>(dec->ops.size());
  p.kc = dec->kc;
  p.head_op = dec->head_op;
  p.head_first = dec->head_first;
  p.chunks_per_token = dec->cpt;
  p.steps = steps;
  p.chunk_addr = reinterpret_cast<const unsigned long long*>(ws + dec->off_chunk_addr);
  p.chunk_bytes = reinterpret_cast<const unsigned*>(ws + dec->off_chunk_bytes);
  p.attn_addr = reinterpret_cast<const unsigned long long*>(ws + dec->off_attn_addr);
  p.attn_bytes = reinterpret_cast<const unsigned*>(ws + dec->off_attn_bytes);
  p.attn_ops = reinterpret_cast<const int32_t*>(ws + dec->off_attn_ops);
  p.n_mla = static_cast<int32_t>(dec->attn_ops.size());
  p.ll = reinterpret_cast<unsigned long long*>(ws + dec->off_ll);
  p.epoch = reinterpret_cast<unsigned*>(ws + dec->off_sync + 4);
  p.d = dec->d;
  p.sm = dec->sm;
  p.head = md.head;
  p.logits = md.logits;
  p.token = md.token;
  p.position = md.position;
  p.seen = md.seen;
  p.history = md.history;
  p.history_len = md.history_len;
  p.sampling = md.sampling;
  p.top_k = md.top_k;
  p.rng = md.rng;
  p.error = error;
  p.feed = feed;
  p.timeout_ns = timeout_ns == 0 ? 1000000000ull : timeout_ns;
  p.trace = dec->trace;
  p.trace_step = dec->trace_step;
  p.flags = flags;
  IVB_CUDA(cudaMemsetAsync(error, 0, 4, s));
  // cooperative: every CTA is resident at once (they wait on one another's flag words)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(dec->R + dec->A);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = dec->smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  IVB_CUDA(cudaLaunchKernelEx(&cfg, p.trace != nullptr ? grid_decode_kernel<true> : grid_decode_kernel<false>, p));
  return IVB_OK;
}

int32_t ivb_decoder_trace(IvbDecoder* dec, uint64_t* buffer, int32_t step) {
  using namespace ivb;
  if (dec == nullptr || step < 0) return fail(IVB_EINVAL, "ivb_decoder_trace: bad argument");
  dec->trace = reinterpret_cast<unsigned long long*>(buffer);
  dec->trace_step = step;
  return IVB_OK;
}

int32_t ivb_decoder_check(IvbDecoder* dec, void* stream) {
  using namespace ivb;
  if (dec == nullptr || dec->ws == nullptr) return fail(IVB_EINVAL, "ivb_decoder_check: decoder not bound");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  IVB_CUDA(cudaStreamSynchronize(s));
  unsigned word = 0;
  IVB_CUDA(cudaMemcpy(&word, dec->ws + dec->off_sync, sizeof(word), cudaMemcpyDeviceToHost));
  if (word == IVB_ECAPACITY) return fail(IVB_ECAPACITY, "the decoder has no free position left");
  if (word == IVB_EINVAL) return fail(IVB_EINVAL, "a token id is out of range for the vocabulary");
  if (word != 0) return fail(static_cast<int32_t>(word), "a bounded wait in the decode kernel gave up (device error word %u)", word);
  return IVB_OK;
}

}  // extern "C"
