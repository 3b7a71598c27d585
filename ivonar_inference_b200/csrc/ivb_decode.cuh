// Whole-GPU decode kernel of libivonar_b200.so: device-side structures and helpers.
//
// One cooperative launch of G CTAs (one per SM) runs the whole token loop: R GEMV CTAs run every
// projection (and the recurrent step of their channels), and one attention CTA per head runs that
// head's latent attention, so each CTA executes a small set of code that stays in the instruction cache.
// Every op of the per-token program is a dependent phase across the GPU: each producer CTA writes
// its slice of the op's output vector as 8-byte words {value, token epoch} into a global buffer
// owned by that op, and each consumer CTA gathers the whole vector by polling those words until
// every one carries the current epoch (the flag travels inside the data word, so one L2 round trip
// both synchronises and delivers; no fence and no counter). Weights reach the CTAs as a per-CTA
// linear stream (laid out once at bind time): a ring of cp.async.bulk copies fed ahead of use, each
// stage completing on an mbarrier, so the weight stream overlaps the handoff latency. Per block:
//   mamba: [norm+quant -> entry rows of my channels (value, gate) and of their head (B, C, dt) -> SSM
//           step of my channels] | out | gate/up | down
//   mla:   [norm+quant -> entry rows (q, latent, k_rope slices)] | attention (one dedicated CTA per
//           head) | out | gate/up | down
// then the LM head with a local top-k per CTA, a merge by group leaders and a final merge that every
// CTA runs identically. Replaces the reference's per-token launch list and its 16-token CUDA graph
// (kernel_decoder.py:179-283, 683-735).
#pragma once

#include "ivb_device.cuh"

namespace ivb {

constexpr int kStages = 6;      // ring stages of a GEMV CTA's weight stream
constexpr int kAttnStages = 2;  // ring stages of an attention CTA (the last two of the ring; the rest holds tiles)

enum OpKind : int32_t {
  OP_ENTRY_MAMBA = 0, OP_ENTRY_MLA = 1, OP_ATTN = 2, OP_OUT = 3, OP_GATE_UP = 4, OP_DOWN = 5, OP_HEAD = 6, OP_MERGE = 7
};
// Where a gathered input vector lands in shared memory.
enum InDst : int32_t { IN_NONE = 0, IN_RESID = 1, IN_VEC = 2, IN_LATENT = 3, IN_CAND = 4, IN_PARTS = 5 };

// One step of the per-token program; identical for every CTA.
struct Op {
  int32_t kind, layer;
  int32_t first_chunk, n_chunks;  // chunks of the weight stream this op consumes (norm chunk, constants chunk, rows)
  int32_t has_norm_chunk, has_const;
  int32_t in_dst;                  // InDst of the gathered input
  int32_t ll_in, ll_in_words;      // input: word offset of the previous op's output buffer and its length (-1: none)
  int32_t ll_out;                  // word offset of this op's output buffer
  int32_t in_n;                    // GEMV input length
  int32_t rows_per, rows_total;    // uniform row partition across the CTAs (attention: the head's kv rows)
  int32_t chunk_rows;              // rows per stream chunk
  int32_t row_bytes, scale_stride, has_bias, lpr_log;
  int32_t has_norm;
  float norm_eps;
  // constants chunk: byte offsets of its arrays
  int32_t c_decay, c_theta, c_skip, c_convw, c_convb;
};

// Device record of one op: its descriptor and a copy of its block's layer description, so one
// prefetch brings every per-op parameter into shared memory.
struct __align__(16) OpRec {
  Op op;
  IvbLayerDesc layer;  // zero for the head
};

struct DecodeDims {
  int32_t vocab, hidden, heads, head_dim, state_dim, latent, rope, nope, dense, max_len, max_top_k;
  int32_t R;                       // GEMV CTAs (ranks 0 .. R-1); ranks R .. R+heads-1 are the attention CTAs
  int32_t cpc;                     // recurrent channels per GEMV CTA (hidden / R, within one head)
  int32_t A;                       // attention CTAs (heads, or 0 without attention blocks)
  int32_t taps;                    // conv taps
  int32_t ssm_v16, ssm_lg_cs;      // recurrent state prefetch: one 16-byte copy per thread; log2(cpc / 2)
  int32_t lpad, rpad;              // latent cache row stride (bytes), k_rope cache row stride (halves)
  int32_t kvpad;                   // key / value cache row stride (floats): head_dim rounded up to 4
  int32_t rb_lat, ss_lat;          // row bytes / scale stride of latent-input matrices
  int32_t tile;                    // cached positions per attention tile
  int32_t group;                   // CTAs per candidate-merge group (the group's first CTA merges)
  int32_t cand_cap;                // candidates one merge can hold in shared memory
  float act_eps, clip;
  float half_dt_min, half_dt_range;
};

// Shared-memory map (byte offsets from the dynamic shared memory base).
struct DecodeSmem {
  int32_t ring, stage_bytes;
  int32_t act, xsum, resid, pub, pub_n, loc, red, xl;  // xl: the attention op's gathered [q_h | latent | k_rope_h]
  int32_t ctab;                    // chunk table of the CTA: [cpt] u64 addresses, then [cpt] u32 sizes
  int32_t cand;                    // offset inside the union region of the gathered candidate arrays (keys, ids)
  int32_t rope_row;                // rope (cos, sin) row of the current position, prefetched by the mla entry op
  int32_t seen;                    // the CTA's slice of the repetition flags, prefetched by the head op
  int32_t u;                       // union region (attention / SSM / sampler)
  int32_t total;
};

struct DecodeParams {
  const OpRec* ops;
  const int32_t* op_rows;          // [n_ops][R] output rows of each CTA
  int32_t n_ops;
  int32_t kc;                      // candidate slots per CTA (>= top-k)
  int32_t head_op;                 // index of the head op (the ops from it on run only when a head is needed)
  int32_t head_first;              // first stream chunk of the head op
  int32_t chunks_per_token;
  int32_t steps;
  const unsigned long long* chunk_addr;  // [R][chunks_per_token] device addresses of the GEMV CTAs' stream chunks
  const unsigned* chunk_bytes;           // [R][chunks_per_token]
  const unsigned long long* attn_addr;   // [heads][n_mla] the attention CTAs' chunks (one per attention op)
  const unsigned* attn_bytes;            // [heads][n_mla]
  const int32_t* attn_ops;               // [n_mla] indices of the attention ops in `ops`
  int32_t n_mla;
  unsigned long long* ll;          // flag-word buffers of all ops (one token's worth, reused every token)
  unsigned* epoch;                 // [1] last token epoch used by any run; flags are epoch + 1, + 2, ...
  DecodeDims d;
  DecodeSmem sm;
  IvbTernary head;                 // original head matrix (embedding rows)
  float* logits;
  int64_t* token;
  int64_t* position;
  uint8_t* seen;
  int64_t* history;
  int32_t history_len;
  const float* sampling;
  const int64_t* top_k;
  uint64_t* rng;
  unsigned* error;
  const int64_t* feed;
  unsigned long long timeout_ns;
  unsigned long long* trace;       // [n_ops][R][8]
  int32_t trace_step;
  int32_t flags;
};

__device__ __forceinline__ int part_lo(int n, int per, int c) { return min(n, c * per); }
__device__ __forceinline__ int part_hi(int n, int per, int c) { return min(n, (c + 1) * per); }

// ---- flag words: {payload in the low 32 bits, token epoch in the high 32 bits} ------------------
// A 64-bit aligned relaxed access at gpu scope is single-copy atomic, so a consumer that sees the
// epoch also sees the payload written with it.
__device__ __forceinline__ void ll_store(unsigned long long* w, unsigned payload, unsigned flag) {
  const unsigned long long v = (static_cast<unsigned long long>(flag) << 32) | payload;
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(w), "l"(v) : "memory");
}
__device__ __forceinline__ void ll_load2(const unsigned long long* w, unsigned long long& a, unsigned long long& b) {
  asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ll_load1(const unsigned long long* w) {
  unsigned long long a;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(a) : "l"(w) : "memory");
  return a;
}

// Producer side: words [base, base + n) of buffer `buf` <- src[0, n) (any CTA threads).
__device__ __forceinline__ void ll_put(unsigned long long* buf, int base, const float* src, int n, unsigned flag) {
  for (int i = threadIdx.x; i < n; i += kThreads) ll_store(buf + base + i, __float_as_uint(src[i]), flag);
}

// Consumer side, every thread of the CTA: dst <- the payloads of words [0, n1) of src1, then [0, n2) of
// src2, then [0, n3) of src3, once every word carries `flag`. The pairs of words are loaded all at once
// (kLLPairs per thread per pass) and only the missing ones are polled again. Bounded: returns false in
// every thread if some word did not arrive within timeout_ns (the verdict is uniform across the CTA).
// The sources are 16-byte aligned; n1 and n2 are even (an odd word may end the last range only).
constexpr int kLLPairs = 9;
__device__ __forceinline__ bool ll_gather3(const unsigned long long* src1, int n1, const unsigned long long* src2, int n2,
                                               const unsigned long long* src3, int n3, unsigned flag, unsigned* dst,
                                               unsigned long long timeout_ns) {
  const int p1 = n1 >> 1, p2 = p1 + (n2 >> 1), pairs = p2 + (n3 >> 1);
  bool late = false;
  for (int base = 0; base < pairs; base += kLLPairs * kThreads) {
    unsigned long long a[kLLPairs], b[kLLPairs];
    const unsigned long long* w[kLLPairs];
#pragma unroll
    for (int j = 0; j < kLLPairs; ++j) {
      const int q = base + j * kThreads + static_cast<int>(threadIdx.x);
      w[j] = q < p1 ? src1 + 2 * q : q < p2 ? src2 + 2 * (q - p1) : src3 + 2 * (q - p2);
      if (q < pairs) {
        ll_load2(w[j], a[j], b[j]);
      } else {
        a[j] = static_cast<unsigned long long>(flag) << 32;
        b[j] = a[j];
      }
    }
    unsigned long long t0 = 0ull;
    unsigned spins = 0u;
    while (!late) {
      bool miss = false;
#pragma unroll
      for (int j = 0; j < kLLPairs; ++j) {
        if (static_cast<unsigned>(a[j] >> 32) != flag || static_cast<unsigned>(b[j] >> 32) != flag) {
          miss = true;
          ll_load2(w[j], a[j], b[j]);
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
    for (int j = 0; j < kLLPairs; ++j) {
      const int q = base + j * kThreads + static_cast<int>(threadIdx.x);
      if (q < pairs) {
        dst[2 * q] = static_cast<unsigned>(a[j]);
        dst[2 * q + 1] = static_cast<unsigned>(b[j]);
      }
    }
  }
  // an odd last word of the last non-empty range
  const int odd_n = n3 > 0 ? n3 : n2 > 0 ? n2 : n1;
  if ((odd_n & 1) && threadIdx.x == 0 && !late) {
    const unsigned long long* last = n3 > 0 ? src3 + n3 - 1 : n2 > 0 ? src2 + n2 - 1 : src1 + n1 - 1;
    unsigned long long v = ll_load1(last);
    const unsigned long long t0 = global_ns();
    while (static_cast<unsigned>(v >> 32) != flag) {
      if (global_ns() - t0 > timeout_ns) {
        late = true;
        break;
      }
      v = ll_load1(last);
    }
    dst[n1 + n2 + n3 - 1] = static_cast<unsigned>(v);
  }
  return !__syncthreads_or(late);
}
__device__ __forceinline__ bool ll_gather2(const unsigned long long* src1, int n1, const unsigned long long* src2, int n2,
                                           unsigned flag, unsigned* dst, unsigned long long timeout_ns) {
  return ll_gather3(src1, n1, src2, n2, src2, 0, flag, dst, timeout_ns);
}
__device__ __forceinline__ bool ll_gather(const unsigned long long* buf, int n, unsigned flag, unsigned* dst,
                                          unsigned long long timeout_ns) {
  return ll_gather3(buf, n, buf, 0, buf, 0, flag, dst, timeout_ns);
}

// ---- weight stream ------------------------------------------------------------------------------
// Lives in shared memory. The producer cursor (issued, p_step, p_chunk) belongs to thread 0; the
// consumers address chunk number `idx` of the run (every thread knows it: the chunks consumed by
// earlier tokens plus the op's first chunk), so no per-thread counter travels between routines.
// What a consumer of the stream needs, held by value (registers or rematerialised constants) so that
// acquiring a chunk does not first chase pointers through shared memory.
struct RingView {
  unsigned long long* full;  // the ring's mbarriers
  unsigned char* ring;       // its first stage
  int stage_bytes;
  unsigned long long timeout_ns;
};

struct Stream {
  unsigned long long* full;  // [NS] mbarriers
  unsigned char* ring;
  int stage_bytes;
  const unsigned long long* caddr;  // this CTA's chunk table (shared copy): device addresses
  const unsigned* cbytes;           // chunk sizes
  int cpt, head_first;       // chunks per token, first chunk of the head (skipped by tokens without one)
  unsigned issued;
  int p_step, p_chunk;       // producer cursor
};

__device__ __forceinline__ bool head_needed(const DecodeParams& p, int step) {
  return (p.flags & (IVB_RUN_SAMPLE | IVB_RUN_HEAD_ALL)) != 0 || step == p.steps - 1;
}
// chunks a token consumes: all of them, or those before the head's when it computes no head
__device__ __forceinline__ int chunks_of_step(const DecodeParams& p, const Stream* s, int step) {
  return head_needed(p, step) ? s->cpt : s->head_first;
}

// thread 0 only, after a CTA barrier that follows the last read of the freed stages (chunks below
// `consumed` are no longer read): queue the chunks of this CTA's stream that follow, into its NS ring stages in turn,
// until `consumed + NS` chunks are issued or the run's steps are exhausted. The cursor and the stream's
// constants are read from shared memory once and kept in registers while the copies are issued (a
// chain of dependent shared-memory accesses per chunk would put hundreds of cycles between an op's end
// and the next op's gather on the CTA that finishes last).
template <int NS = kStages>
__device__ __forceinline__ void stream_refill(const DecodeParams& p, Stream* s, unsigned consumed) {
  unsigned issued = s->issued;
  int p_step = s->p_step, p_chunk = s->p_chunk;
  const int steps = p.steps;
  if (issued >= consumed + NS || p_step >= steps) return;
  const int cpt = s->cpt, head_first = s->head_first, stage_bytes = s->stage_bytes;
  unsigned long long* const full = s->full;
  unsigned char* const ring = s->ring;
  const unsigned long long* const caddr = s->caddr;
  const unsigned* const cbytes = s->cbytes;
  while (issued < consumed + NS && p_step < steps) {
    if (p_chunk == head_first && !head_needed(p, p_step)) {  // a token without a head skips its chunks
      p_chunk = 0;
      if (++p_step >= steps) break;
    }
    const unsigned bytes = cbytes[p_chunk];
    const int stage = static_cast<int>(issued % NS);
    mbar_expect_tx(full + stage, bytes);  // the stage is only ever written by the copy engine: no proxy fence
    bulk_copy(ring + static_cast<size_t>(stage) * stage_bytes, reinterpret_cast<const void*>(caddr[p_chunk]), bytes, full + stage);
    ++issued;
    if (++p_chunk == cpt) {
      p_chunk = 0;
      ++p_step;
    }
  }
  s->issued = issued;
  s->p_step = p_step;
  s->p_chunk = p_chunk;
}

// Bounded wait on an mbarrier phase by one thread; true when the phase completed.
__device__ __forceinline__ bool mbar_wait_bounded(unsigned long long* bar, unsigned parity, unsigned long long timeout_ns) {
  unsigned long long t0 = 0ull;
  unsigned spins = 0u;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 255u) == 0u) {
      const unsigned long long t = global_ns();
      if (t0 == 0ull) t0 = t;
      else if (t - t0 > timeout_ns) return false;
    }
  }
  return true;
}

// every thread: wait until chunk `idx` of the run has landed in its ring stage (each thread's own
// mbarrier wait makes the copied bytes visible to it; no CTA barrier). Returns the stage base, or
// nullptr when this thread's bounded wait ran out (the op reports it after its closing barrier).
template <int NS = kStages>
__device__ __forceinline__ const unsigned char* stream_acquire(const RingView& v, unsigned idx) {
  const int stage = idx % NS;
  const unsigned parity = (idx / NS) & 1u;
  if (!mbar_wait_bounded(v.full + stage, parity, v.timeout_ns)) return nullptr;
  return v.ring + static_cast<size_t>(stage) * v.stage_bytes;
}


// ---- GEMV rows from a ring stage ----------------------------------------------------------------
// dp4a with unsigned weight bytes and signed activation bytes.
__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Activations of one 64-input chunk in registers: q[k] are the four act words of weight word k.
struct ActChunk {
  int4 q[4];
  int xsum;
};

// The chunk sum of the codes: xsum[u], or the two half sums xhalf[2u], xhalf[2u + 1], or (both null)
// computed here with sixteen dp4a with ones.
__device__ __forceinline__ ActChunk load_act_chunk(const int8_t* act, const int* xsum, int u, const int* xhalf = nullptr) {
  ActChunk c;
  const int rot = (u >> 1) & 3;
  const char* base = reinterpret_cast<const char*>(act) + (u << 6);
#pragma unroll
  for (int k = 0; k < 4; ++k) c.q[k] = *reinterpret_cast<const int4*>(base + (((k + rot) & 3) << 4));
  if (xsum != nullptr) {
    c.xsum = xsum[u];
  } else if (xhalf != nullptr) {
    c.xsum = xhalf[2 * u] + xhalf[2 * u + 1];
  } else {
    int t = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      t = __dp4a(c.q[k].x, 0x01010101, t);
      t = __dp4a(c.q[k].y, 0x01010101, t);
      t = __dp4a(c.q[k].z, 0x01010101, t);
      t = __dp4a(c.q[k].w, 0x01010101, t);
    }
    c.xsum = t;
  }
  return c;
}

// 64 times the exact integer sum over the chunk of (code - 1) * q8. The two-bit field f of every weight
// byte is masked in place (value code << 2f) and dotted with the activations of field f; the partial
// sums are combined with shift-adds (64 s0 + 16 s1 + 4 s2 + s3 - 64 xsum), and the factor 64 is folded
// into the group scale by the caller (|result| < 2^23, so its float is exact).
__device__ __forceinline__ int chunk_dot64(const uint4 w, const ActChunk& a) {
  const unsigned ws[4] = {w.x, w.y, w.z, w.w};
  int s0 = 0, s1 = 0, s2 = 0, s3 = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    s0 = dp4a_us(ws[k] & 0x03030303u, a.q[k].x, s0);
    s1 = dp4a_us(ws[k] & 0x0C0C0C0Cu, a.q[k].y, s1);
    s2 = dp4a_us(ws[k] & 0x30303030u, a.q[k].z, s2);
    s3 = dp4a_us(ws[k] & 0xC0C0C0C0u, a.q[k].w, s3);
  }
  return ((((s0 << 2) + s1) << 2) + s2) * 4 + s3 - (a.xsum << 6);
}

// What rows_generic does with a finished row value v (row r of the chunk): store it to out[r] (shared,
// for an epilogue that needs every row), or publish it as a flag word: resid[r] + v at ll[r] (out and
// down projections), v at ll[r] (mla entry), or silu(v_r) * v_{r+1} at ll[r / 2] for even r (gate/up
// rows interleaved; the two rows' lane groups sit in one warp, lg <= 4).
enum RowsEpi { EPI_STORE = 0, EPI_RESID = 1, EPI_PUBLISH = 2, EPI_SWIGLU = 3 };

// rows_generic with the lane geometry fixed at compile time (2^LG lanes per row, KPL chunks per lane,
// RPT rows per lane group in one pass, interleaved): every thread of the CTA runs every pass (a lane
// group past the last row recomputes row k - 1 and stores nothing), so the lane butterflies are
// full-warp shuffles of a fixed length; each chunk's product has its own accumulator (added in chunk
// order at the end), so the chunk dots of a lane run side by side.
template <int LG, int KPL, int RPT>
__device__ __forceinline__ void rows_ct(const unsigned char* stage, int k, int row_bytes, int sstride, int has_bias, float act_scale,
                                        const int8_t* act, const int* xhalf, int in_n, float* out, int epi, unsigned long long* ll,
                                        const float* resid, unsigned flag) {
  constexpr int kLpr = 1 << LG, kRpi = kThreads >> LG;
  const int chunks = (in_n + 63) >> 6;
  const int sub = threadIdx.x & (kLpr - 1), grp = threadIdx.x >> LG;
  ActChunk a[KPL];
  bool have[KPL];
#pragma unroll
  for (int j = 0; j < KPL; ++j) {
    const int u = sub + (j << LG);
    have[j] = u < chunks;
    if (have[j]) {
      a[j] = load_act_chunk(act, nullptr, u, xhalf);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) a[j].q[q] = make_int4(0, 0, 0, 0);
      a[j].xsum = 0;
    }
  }
  const uint16_t* scales = reinterpret_cast<const uint16_t*>(stage + static_cast<size_t>(k) * row_bytes);
  const float* bias = reinterpret_cast<const float*>(stage + static_cast<size_t>(k) * row_bytes + round16(k * sstride * 2));
  const int passes = (k + kRpi * RPT - 1) / (kRpi * RPT);
  for (int pass = 0; pass < passes; ++pass) {
    float v[RPT];
#pragma unroll
    for (int t = 0; t < RPT; ++t) {
      const int rr = min(pass * kRpi * RPT + t * kRpi + grp, k - 1);
      const uint4* wr = reinterpret_cast<const uint4*>(stage + rr * row_bytes);
      const uint16_t* srow = scales + rr * sstride;
      float part[KPL];
#pragma unroll
      for (int j = 0; j < KPL; ++j) {
        const int u = sub + (j << LG);
        part[j] = have[j] ? static_cast<float>(chunk_dot64(wr[u], a[j])) * (h2f(srow[u >> 1]) * (1.0f / 64.0f)) : 0.0f;
      }
      float acc = part[0];
#pragma unroll
      for (int j = 1; j < KPL; ++j) acc += part[j];
      v[t] = acc;
    }
#pragma unroll
    for (int off = 1; off < kLpr; off <<= 1)
#pragma unroll
      for (int t = 0; t < RPT; ++t) v[t] += __shfl_xor_sync(kFull, v[t], off);
#pragma unroll
    for (int t = 0; t < RPT; ++t) {
      const int r = pass * kRpi * RPT + t * kRpi + grp;
      const bool valid = r < k;
      const int rr = valid ? r : k - 1;
      const float x = has_bias ? v[t] * act_scale + bias[rr] : v[t] * act_scale;
      if (epi == EPI_SWIGLU) {
        const float up = __shfl_down_sync(kFull, x, kLpr);  // row r + 1 (up) is the next lane group of the warp
        if (valid && sub == 0 && (r & 1) == 0) ll_store(ll + (r >> 1), __float_as_uint(silu_f(x) * up), flag);
      } else if (valid && sub == 0) {
        if (epi == EPI_STORE) out[r] = x;
        else if (epi == EPI_RESID) ll_store(ll + r, __float_as_uint(resid[r] + x), flag);
        else ll_store(ll + r, __float_as_uint(x), flag);
      }
    }
  }
}

// Rows [0, k) of one stream chunk laid out [k x row_bytes packed][k x sstride fp16 (16B pad)][k x fp32
// bias] against the quantised input `act` (transposed GEMV layout, in_n inputs): 2^lg lanes per row
// (lg <= 5), lane `sub` owning the 64-input chunks sub + j * 2^lg (j < 4, so in_n <= 256 * 2^lg), their
// activations held in registers; every row is one chain of fmaf over the lane's chunks followed by
// an xor butterfly over the lanes, then the epilogue `epi`. The plan picks lg per op so that the CTA's
// rows take one pass where the registers allow. One small routine serves every GEMV of the decode kernel.
constexpr int kRowsKPL = 4;
__device__ __forceinline__ void rows_generic(const unsigned char* stage, int k, int row_bytes, int sstride, int has_bias,
                                             float act_scale, const int8_t* act, const int* xhalf, int in_n, int lg, float* out,
                                             int epi, unsigned long long* ll, const float* resid, unsigned flag) {
  const int lpr = 1 << lg, rpi = kThreads >> lg;
  const int chunks = (in_n + 63) >> 6;
  const int sub = threadIdx.x & (lpr - 1);
  if (static_cast<int>(threadIdx.x >> lg) >= k) return;  // lanes without a row in any pass (rpi > k)
  ActChunk a[kRowsKPL];
  bool have[kRowsKPL];
#pragma unroll
  for (int j = 0; j < kRowsKPL; ++j) {
    const int u = sub + (j << lg);
    have[j] = u < chunks;
    if (have[j]) {
      a[j] = load_act_chunk(act, nullptr, u, xhalf);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) a[j].q[q] = make_int4(0, 0, 0, 0);
      a[j].xsum = 0;
    }
  }
  const uint16_t* scales = reinterpret_cast<const uint16_t*>(stage + static_cast<size_t>(k) * row_bytes);
  const float* bias = reinterpret_cast<const float*>(stage + static_cast<size_t>(k) * row_bytes + round16(k * sstride * 2));
  const unsigned mask = lpr >= 32 ? kFull : (((1u << lpr) - 1u) << (threadIdx.x & 31 & ~(lpr - 1)));
#pragma unroll 1
  for (int base = 0; base < k; base += rpi) {
    const int r = base + (static_cast<int>(threadIdx.x) >> lg);
    if (r >= k) break;  // the row group's lanes leave together
    const uint4* wr = reinterpret_cast<const uint4*>(stage + static_cast<size_t>(r) * row_bytes);
    const uint16_t* srow = scales + r * sstride;
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < kRowsKPL; ++j) {
      const int u = sub + (j << lg);
      if (have[j]) acc = fmaf(static_cast<float>(chunk_dot64(wr[u], a[j])), h2f(srow[u >> 1]) * (1.0f / 64.0f), acc);
    }
    for (int off = 1; off < lpr; off <<= 1) acc += __shfl_xor_sync(mask, acc, off);
    const float v = has_bias ? acc * act_scale + bias[r] : acc * act_scale;
    if (epi == EPI_SWIGLU) {
      // rows r (gate, even) and r + 1 (up) are adjacent lane groups of one warp; k is even
      const unsigned pmask = 2 * lpr >= 32 ? kFull : ((1u << (2 * lpr)) - 1u) << (threadIdx.x & 31 & ~(2 * lpr - 1));
      const float up = __shfl_down_sync(pmask, v, lpr);
      if (sub == 0 && (r & 1) == 0) ll_store(ll + (r >> 1), __float_as_uint(silu_f(v) * up), flag);
    } else if (sub == 0) {
      if (epi == EPI_STORE) out[r] = v;
      else if (epi == EPI_RESID) ll_store(ll + r, __float_as_uint(resid[r] + v), flag);
      else ll_store(ll + r, __float_as_uint(v), flag);
    }
  }
}

// The row routine the decode kernel runs on a chunk of k rows: the compile-time geometries for the
// Nano shapes (1024 inputs: 16 lanes per row for up to 16 rows, 8 lanes x 2 rows for up to 64, 8 lanes
// x 8 rows for up to 256; 256 inputs: 4 lanes x 2 rows for up to 128; 2049-4096 inputs and up to 8 rows
// outside gate/up: 32 lanes), rows_generic with 2^lg lanes per row for every other shape.
__device__ __forceinline__ void rows_decode(const unsigned char* stage, int k, int row_bytes, int sstride, int has_bias,
                                            float act_scale, const int8_t* act, const int* xhalf, int in_n, int lg, float* out,
                                            int epi, unsigned long long* ll, const float* resid, unsigned flag) {
  const int chunks = (in_n + 63) >> 6;
  if (chunks == 16) {
    if (k <= 16) return rows_ct<4, 1, 1>(stage, k, row_bytes, sstride, has_bias, act_scale, act, xhalf, in_n, out, epi, ll, resid, flag);
    if (k <= 64) return rows_ct<3, 2, 2>(stage, k, row_bytes, sstride, has_bias, act_scale, act, xhalf, in_n, out, epi, ll, resid, flag);
    if (k <= 256) return rows_ct<3, 2, 8>(stage, k, row_bytes, sstride, has_bias, act_scale, act, xhalf, in_n, out, epi, ll, resid, flag);
  } else if (chunks == 4 && k <= 128 && epi != EPI_SWIGLU) {  // 256 inputs: the attention's kv rows
    return rows_ct<2, 1, 2>(stage, k, row_bytes, sstride, has_bias, act_scale, act, xhalf, in_n, out, epi, ll, resid, flag);
  } else if (chunks > 32 && chunks <= 64 && k <= 8 && epi != EPI_SWIGLU) {
    return rows_ct<5, 2, 1>(stage, k, row_bytes, sstride, has_bias, act_scale, act, xhalf, in_n, out, epi, ll, resid, flag);
  }
  rows_generic(stage, k, row_bytes, sstride, has_bias, act_scale, act, xhalf, in_n, lg, out, epi, ll, resid, flag);
}

// ---- top-k selection (radix select over order-preserving keys) ----------------------------------
struct TopkScratch {
  unsigned* hist;  // [kWarps * 256]
  int* misc;       // [16]
};

static __device__ __noinline__ void topk_digit(const TopkScratch ts, const unsigned* keys, int n, int shift, unsigned prefix,
                                              unsigned mask, int remaining) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int b = tid; b < kWarps * 256; b += kThreads) ts.hist[b] = 0u;
  __syncthreads();
  unsigned* wh = ts.hist + warp * 256;
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
  const int dgt = 255 - tid;
  unsigned cnt = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) cnt += ts.hist[w * 256 + dgt];
  unsigned incl = cnt;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const unsigned o = __shfl_up_sync(kFull, incl, off);
    if (lane >= off) incl += o;
  }
  if (lane == 31) ts.misc[warp] = static_cast<int>(incl);
  __syncthreads();
  unsigned carry = 0;
  for (int w = 0; w < warp; ++w) carry += static_cast<unsigned>(ts.misc[w]);
  incl += carry;
  const unsigned above = incl - cnt;
  if (cnt > 0 && static_cast<int>(above) < remaining && remaining <= static_cast<int>(above + cnt)) {
    ts.misc[8] = dgt;
    ts.misc[9] = remaining - static_cast<int>(above);
  }
  __syncthreads();
}

// The K best of keys[0, n) by (key desc, id asc); ids[i] (or id_base + i when ids == nullptr) must
// increase with i among equal keys. Writes them sorted into out_key / out_id (K <= kMaxTopK).
static __device__ __noinline__ void topk_sorted(const unsigned* keys, const int* ids, int id_base, int n, int K, const TopkScratch ts,
                                   unsigned* ck, int* ci, unsigned* out_key, int* out_id) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  unsigned prefix = 0u, mask = 0u;
  int remaining = K;
  for (int shift = 24; shift >= 0; shift -= 8) {
    topk_digit(ts, keys, n, shift, prefix, mask, remaining);
    prefix |= static_cast<unsigned>(ts.misc[8]) << shift;  // the digit of the K-th key and what is left below it
    mask |= 255u << shift;
    remaining = ts.misc[9];
    __syncthreads();
  }
  const unsigned thr = prefix;
  if (tid == 0) {
    ts.misc[10] = 0;
    ts.misc[11] = 0;
  }
  __syncthreads();
  for (int i = tid; i < n; i += kThreads) {
    const unsigned k = keys[i];
    if (k > thr) {
      const int slot = atomicAdd(&ts.misc[10], 1);
      ck[slot] = k;
      ci[slot] = ids ? ids[i] : id_base + i;
    } else if (k == thr) {
      atomicAdd(&ts.misc[11], 1);
    }
  }
  __syncthreads();
  const int greater = ts.misc[10];
  if (ts.misc[11] == remaining) {
    if (tid == 0) ts.misc[12] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += kThreads) {
      if (keys[i] == thr) {
        const int slot = greater + atomicAdd(&ts.misc[12], 1);
        ck[slot] = thr;
        ci[slot] = ids ? ids[i] : id_base + i;
      }
    }
  } else if (warp == 0) {
    int taken = 0;
    for (int base = 0; base < n && taken < remaining; base += 32) {
      const int i = base + lane;
      const bool eq = i < n && keys[i] == thr;
      const unsigned bal = __ballot_sync(kFull, eq);
      const int rank = __popc(bal & ((1u << lane) - 1u));
      if (eq && taken + rank < remaining) {
        ck[greater + taken + rank] = thr;
        ci[greater + taken + rank] = ids ? ids[i] : id_base + i;
      }
      taken += __popc(bal);
    }
  }
  __syncthreads();
  for (int c = tid; c < K; c += kThreads) {
    const unsigned kc = ck[c];
    const int ic = ci[c];
    int rank = 0;
    for (int o = 0; o < K; ++o) {
      const unsigned ko = ck[o];
      rank += (ko > kc || (ko == kc && ci[o] < ic)) ? 1 : 0;
    }
    out_key[rank] = kc;
    out_id[rank] = ic;
  }
  __syncthreads();
}

// p_c = exp(s_c - s_0) over sorted keys, canonical CDF (32-candidate Hillis-Steele chunks, carries
// in order), u = philox(key, counter), token = #(cdf <= u * total) clamped to K - 1.
static __device__ __noinline__ int draw_token(const unsigned* sorted_key, const int* sorted_id, int K, float* cdf, float* red,
                                 uint64_t key, uint64_t counter) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float top = key_value(sorted_key[0]);
  for (int c = tid; c < K; c += kThreads) cdf[c] = sample_exp(key_value(sorted_key[c]) - top);
  __syncthreads();
  if (warp == 0) {
    float carry = 0.0f;
    for (int base = 0; base < K; base += 32) {
      const int c = base + lane;
      float v = c < K ? cdf[c] : 0.0f;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float o = __shfl_up_sync(kFull, v, off);
        if (lane >= off) v += o;
      }
      if (c < K) cdf[c] = carry + v;
      carry = carry + __shfl_sync(kFull, v, 31);
    }
  }
  __syncthreads();
  const float uval = fminf(philox_uniform(key, counter), 0.99999994f);
  const float target = uval * cdf[K - 1];
  float below = 0.0f;
  for (int c = tid; c < K; c += kThreads) below += cdf[c] <= target ? 1.0f : 0.0f;
  const int chosen = min(static_cast<int>(block_sum(below, red)), K - 1);
  return sorted_id[chosen];
}

}  // namespace ivb

