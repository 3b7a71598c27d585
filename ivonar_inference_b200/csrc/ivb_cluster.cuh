// Cluster decode kernel of libivonar_b200.so.
//
// One thread-block cluster of R CTAs (R = 16 for the Nano shape, one attention/SSM head per CTA)
// runs the whole token loop. Activations move between CTAs through distributed shared memory: each
// CTA publishes its slice of a vector in its own shared memory, a hardware cluster barrier orders
// the exchange, and consumers read every slice with ld.shared::cluster. Weights reach the CTAs as a
// per-CTA linear stream (laid out once at bind time): a 3-stage ring of cp.async.bulk copies fed
// ahead of use, each stage completing on an mbarrier. Per block the critical path is
//   mamba: [norm+quant -> entry rows of my heads -> SSM step] | out | gate/up | down
//   mla:   [norm+quant -> entry rows (q, k_rope of my heads, my latent rows)] | attention | out | gate/up | down
// with one cluster barrier after each bracket; the head and a distributed top-k sampler end the token.
// Replaces the reference's per-token launch list and its 16-token CUDA graph
// (kernel_decoder.py:179-283, 683-735).
#pragma once

#include "ivb_device.cuh"

namespace ivb {

constexpr int kMaxCluster = 16;
constexpr int kStages = 3;

enum OpKind : int32_t { OP_ENTRY_MAMBA = 0, OP_ENTRY_MLA = 1, OP_ATTN = 2, OP_OUT = 3, OP_GATE_UP = 4, OP_DOWN = 5, OP_HEAD = 6 };
enum Gather : int32_t { G_NONE = 0, G_RESID = 1, G_VEC = 2, G_LATENT = 3 };
// Buffers that other CTAs fill with st.async pushes; each has a transaction-count mbarrier.
enum XBuf : int32_t { XB_RESID = 0, XB_VEC = 1, XB_LATENT = 2, XB_CAND = 3, XB_COUNT = 4, XB_NONE = -1 };

// One step of the per-token program; identical for every CTA of the cluster.
struct Op {
  int32_t kind, layer;
  int32_t first_chunk, n_chunks;  // chunks of the weight stream this op consumes (constants chunk first)
  int32_t has_const;
  int32_t gather;                  // what is gathered from the cluster before the op runs
  int32_t gather_n, gather_per;    // input vector length and per-CTA slice length of its producer
  int32_t push_per;                // entry of an mla block: latent rows per CTA (output slice stride)
  int32_t in_buf;                  // input buffer filled by the previous op's pushes (XB_*), or XB_NONE
  int32_t in_bytes;                // bytes of that fill (all producers together)
  int32_t in_n;                    // GEMV input length
  int32_t rows_per, rows_total;    // uniform row partition across the cluster
  int32_t chunk_rows;              // rows per stream chunk
  int32_t row_bytes, scale_stride, has_bias, lpr_log;
  int32_t epilogue;
  int32_t has_norm;
  float norm_eps;
  // constants chunk: byte offsets of its arrays
  int32_t c_norm, c_decay, c_theta, c_skip, c_convw, c_convb;
  int32_t c_wkn, c_skn, c_bkn, c_wv, c_sv, c_bv;
};

// Device record of one op: its descriptor and a copy of its block's layer description, so one
// prefetch brings every per-op parameter into shared memory.
struct __align__(16) OpRec {
  Op op;
  IvbLayerDesc layer;  // zero for the head
};

struct ClusterDims {
  int32_t vocab, hidden, heads, head_dim, state_dim, latent, rope, nope, dense, max_len, max_top_k;
  int32_t R, hpc;                  // cluster size, heads per CTA
  int32_t taps;                    // conv taps
  int32_t lpad, rpad;              // latent cache row stride (bytes), k_rope cache row stride (halves)
  int32_t rb_lat, ss_lat;          // row bytes / scale stride of latent-input matrices
  int32_t tile;                    // cached positions per attention tile
  float act_eps, clip;
  float half_dt_min, half_dt_range;
};

// Shared-memory map (byte offsets from the dynamic shared memory base).
struct ClusterSmem {
  int32_t ring, stage_bytes;
  int32_t xv, act, xsum, resid, pub, pub_n, loc, red, xl;
  int32_t ctab;                    // chunk table of the CTA: [cpt] u64 offsets, then [cpt] u32 sizes
  int32_t cand;                    // offset inside the union region of the merge arrays (keys, ids) the head pushes into
  int32_t rope_row;                // rope (cos, sin) row of the current position, prefetched by the mla entry op
  int32_t seen;                    // the CTA's slice of the repetition flags, prefetched by the head op
  int32_t u;                       // union region (attention / sampler)
  int32_t total;
};

struct ClusterParams {
  const OpRec* ops;
  const int32_t* op_rows;          // [n_ops][R] output rows of each CTA
  int32_t n_ops;
  int32_t kc;                      // candidate slots per CTA (>= top-k)
  int32_t head_first;              // first stream chunk of the head op
  int32_t chunks_per_token;
  int32_t steps;
  const unsigned long long* chunk_off;  // [R][chunks_per_token] byte offsets into the stream
  const unsigned* chunk_bytes;          // [R][chunks_per_token]
  const unsigned char* stream;
  ClusterDims d;
  ClusterSmem sm;
  const IvbLayerDesc* layers;
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
  unsigned* cand_key;              // [R][K] local top-k candidates of each CTA
  int* cand_id;
  int* cand_n;                     // [R]
  unsigned* error;
  const int64_t* feed;
  unsigned long long timeout_ns;
  unsigned long long* trace;       // [n_ops][R][8]
  int32_t trace_step;
  int32_t flags;
};

// ---- cluster primitives -------------------------------------------------------------------------
__device__ __forceinline__ unsigned cluster_rank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ unsigned map_rank(const void* local, unsigned rank) {
  unsigned r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(local)), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_cluster_f32(unsigned addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_cluster_f32(unsigned addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_v4(unsigned addr, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}
// st.async into another CTA's shared memory; the bytes complete a transaction on that CTA's mbarrier.
__device__ __forceinline__ void st_async_v4(unsigned addr, float4 v, unsigned mbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(addr),
               "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(mbar)
               : "memory");
}
__device__ __forceinline__ void st_async_b32(unsigned addr, unsigned v, unsigned mbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(addr), "r"(v), "r"(mbar)
               : "memory");
}
__device__ __forceinline__ void atom_min_cluster_u32(unsigned addr, unsigned v) {
  asm volatile("red.shared::cluster.min.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ int part_lo(int n, int per, int c) { return min(n, c * per); }
__device__ __forceinline__ int part_hi(int n, int per, int c) { return min(n, (c + 1) * per); }

// ---- weight stream ------------------------------------------------------------------------------
struct Stream {
  unsigned long long* full;  // [kStages] mbarriers
  unsigned char* ring;
  int stage_bytes;
  const unsigned long long* coff;  // this CTA's chunk table (shared copy): byte offsets into the stream
  const unsigned* cbytes;          // chunk sizes
  unsigned consumed, issued;
  int p_step, p_chunk;       // producer cursor
};

__device__ __forceinline__ bool head_needed(const ClusterParams& p, int step) {
  return (p.flags & (IVB_RUN_SAMPLE | IVB_RUN_HEAD_ALL)) != 0 || step == p.steps - 1;
}

// thread 0 only: queue the next chunk of this CTA's stream into the next ring stage
__device__ __forceinline__ void stream_issue(const ClusterParams& p, Stream& s, unsigned rank) {
  if (s.p_step >= p.steps) return;
  if (s.p_chunk == p.head_first && !head_needed(p, s.p_step)) {
    s.p_chunk = 0;
    if (++s.p_step >= p.steps) return;
  }
  const unsigned bytes = s.cbytes[s.p_chunk];
  const int stage = s.issued % kStages;
  unsigned long long* bar = s.full + stage;
  mbar_expect_tx(bar, bytes);  // the stage is only ever written by the copy engine: no proxy fence
  bulk_copy(s.ring + static_cast<size_t>(stage) * s.stage_bytes, p.stream + s.coff[s.p_chunk], bytes, bar);
  ++s.issued;
  if (++s.p_chunk == p.chunks_per_token) {
    s.p_chunk = 0;
    ++s.p_step;
  }
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

// all threads: wait until the next chunk has landed; returns its stage base, or nullptr in every
// thread when any thread's bounded wait ran out (the verdict is uniform across the CTA)
__device__ __forceinline__ const unsigned char* stream_acquire(const ClusterParams& p, Stream& s) {
  const int stage = s.consumed % kStages;
  const unsigned parity = (s.consumed / kStages) & 1u;
  const bool late = !mbar_wait_bounded(s.full + stage, parity, p.timeout_ns);
  if (__syncthreads_or(late)) return nullptr;
  return s.ring + static_cast<size_t>(stage) * s.stage_bytes;
}

// all threads: the chunk is no longer read; refill its stage with a later chunk
__device__ __forceinline__ void stream_release(const ClusterParams& p, Stream& s, unsigned rank) {
  __syncthreads();
  if (threadIdx.x == 0) stream_issue(p, s, rank);
  ++s.consumed;
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

// xsum == nullptr: the chunk sum of the codes is computed here (sixteen dp4a with ones).
__device__ __forceinline__ ActChunk load_act_chunk(const int8_t* act, const int* xsum, int u) {
  ActChunk c;
  const int rot = (u >> 1) & 3;
  const char* base = reinterpret_cast<const char*>(act) + (u << 6);
#pragma unroll
  for (int k = 0; k < 4; ++k) c.q[k] = *reinterpret_cast<const int4*>(base + (((k + rot) & 3) << 4));
  if (xsum != nullptr) {
    c.xsum = xsum[u];
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

// Exact integer sum over the chunk of (code - 1) * q8. The two-bit field f of every weight byte is
// masked in place (value code << 2f) and dotted with the activations of field f; the four partial
// sums are exact multiples of 1, 4, 16 and 64, so the shifts below are exact.
__device__ __forceinline__ int chunk_dot_regs(const uint4 w, const ActChunk& a) {
  const unsigned ws[4] = {w.x, w.y, w.z, w.w};
  int s0 = 0, s1 = 0, s2 = 0, s3 = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    s0 = dp4a_us(ws[k] & 0x03030303u, a.q[k].x, s0);
    s1 = dp4a_us(ws[k] & 0x0C0C0C0Cu, a.q[k].y, s1);
    s2 = dp4a_us(ws[k] & 0x30303030u, a.q[k].z, s2);
    s3 = dp4a_us(ws[k] & 0xC0C0C0C0u, a.q[k].w, s3);
  }
  return (s0 + (s1 >> 2)) + ((s2 >> 4) + (s3 >> 6)) - a.xsum;
}

// The same sum times 64, combined with shift-adds (64 s0 + 16 s1 + 4 s2 + s3 - 64 xsum); exact, and
// the factor 64 is folded into the group scale by the caller (|result| < 2^23, so its float is exact).
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

// rows [0, k) of a chunk laid out [k x row_bytes packed][k x scale_stride fp16 (16B pad)][k x fp32 bias]
// Lane group of 2^lpr_log lanes per row; lane `sub` owns chunks sub + j * 2^lpr_log (j < KPL), whose
// activations stay in registers for all rows. Every thread runs RPT rows per pass. Results of row r
// go to out[r] (after the lane reduction).
template <int KPL, int RPT>
__device__ __forceinline__ void chunk_rows_kpl(const Op& op, const unsigned char* stage, int k, const int8_t* act,
                                               const int* xsum, float act_scale, float* out) {
  const int tid = threadIdx.x;
  const int lg = op.lpr_log;
  const int lpr = 1 << lg;
  const int rpi = kThreads >> lg;
  const int chunks = (op.in_n + 63) >> 6;
  const int row_bytes = op.row_bytes, sstride = op.scale_stride;  // op lives in shared memory
  const bool has_bias = op.has_bias != 0;
  const int sub = tid & (lpr - 1);
  ActChunk a[KPL];
  bool have[KPL];
#pragma unroll
  for (int j = 0; j < KPL; ++j) {
    const int u = sub + (j << lg);
    have[j] = u < chunks;
    if (have[j]) a[j] = load_act_chunk(act, nullptr, u);
  }
  const uint16_t* scales = reinterpret_cast<const uint16_t*>(stage + static_cast<size_t>(k) * row_bytes);
  const float* bias = reinterpret_cast<const float*>(stage + static_cast<size_t>(k) * row_bytes + round16(k * sstride * 2));
  for (int base = 0; base < k; base += RPT * rpi) {
    int r[RPT];
    bool v[RPT];
    uint4 w[RPT][KPL];
#pragma unroll
    for (int t = 0; t < RPT; ++t) {
      r[t] = base + t * rpi + (tid >> lg);
      v[t] = r[t] < k;
      const uint4* wr = reinterpret_cast<const uint4*>(stage + static_cast<size_t>(r[t]) * row_bytes);
#pragma unroll
      for (int j = 0; j < KPL; ++j) {
        const int u = sub + (j << lg);
        w[t][j] = (have[j] && v[t]) ? wr[u] : make_uint4(0u, 0u, 0u, 0u);
      }
    }
    float acc[RPT];
#pragma unroll
    for (int t = 0; t < RPT; ++t) {
      acc[t] = 0.0f;
#pragma unroll
      for (int j = 0; j < KPL; ++j) {
        const int u = sub + (j << lg);
        if (have[j] && v[t])
          acc[t] = fmaf(static_cast<float>(chunk_dot_regs(w[t][j], a[j])), h2f(scales[r[t] * sstride + (u >> 1)]),
                        acc[t]);
      }
    }
    for (int off = 1; off < lpr; off <<= 1) {
#pragma unroll
      for (int t = 0; t < RPT; ++t) acc[t] += __shfl_xor_sync(kFull, acc[t], off);
    }
    if (sub == 0) {
#pragma unroll
      for (int t = 0; t < RPT; ++t)
        if (v[t]) out[r[t]] = has_bias ? acc[t] * act_scale + bias[r[t]] : acc[t] * act_scale;
    }
  }
}

// Compile-time lane geometry for the common shapes: LG = log2 lanes per row, KPL chunks per lane,
// RPT rows per thread per pass. The lane's activation chunks (a, have) are loaded once per op by
// load_act_ct and stay in registers for every stage of the op.
template <int LG, int KPL>
__device__ __forceinline__ void load_act_ct(const int8_t* act, int chunks, ActChunk (&a)[KPL], bool (&have)[KPL]) {
  const int sub = threadIdx.x & ((1 << LG) - 1);
#pragma unroll
  for (int j = 0; j < KPL; ++j) {
    const int u = sub + (j << LG);
    have[j] = u < chunks;
    if (have[j]) {
      a[j] = load_act_chunk(act, nullptr, u);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) a[j].q[q] = make_int4(0, 0, 0, 0);
      a[j].xsum = 0;
    }
  }
}

template <int LG, int KPL, int RPT>
__device__ __forceinline__ void rows_stage_ct(const ActChunk (&a)[KPL], const bool (&have)[KPL], const unsigned char* stage,
                                              int k, int row_bytes, int sstride, bool has_bias, float act_scale, float* out) {
  constexpr int LPR = 1 << LG, RPI = kThreads >> LG;
  const int tid = threadIdx.x, sub = tid & (LPR - 1);
  const uint16_t* scales = reinterpret_cast<const uint16_t*>(stage + static_cast<size_t>(k) * row_bytes);
  const float* bias = reinterpret_cast<const float*>(stage + static_cast<size_t>(k) * row_bytes + round16(k * sstride * 2));
  for (int base = 0; base < k; base += RPT * RPI) {
    int r[RPT];
    uint4 w[RPT][KPL];
#pragma unroll
    for (int t = 0; t < RPT; ++t) {
      r[t] = base + t * RPI + (tid >> LG);
      const uint4* wr = reinterpret_cast<const uint4*>(stage + static_cast<size_t>(min(r[t], k - 1)) * row_bytes);
#pragma unroll
      for (int j = 0; j < KPL; ++j) w[t][j] = have[j] ? wr[sub + (j << LG)] : make_uint4(0u, 0u, 0u, 0u);
    }
    float acc[RPT];
#pragma unroll
    for (int t = 0; t < RPT; ++t) {
      acc[t] = 0.0f;
      const uint16_t* srow = scales + min(r[t], k - 1) * sstride;
#pragma unroll
      for (int j = 0; j < KPL; ++j) {
        const float sc = have[j] ? h2f(srow[(sub + (j << LG)) >> 1]) * (1.0f / 64.0f) : 0.0f;
        acc[t] = fmaf(static_cast<float>(chunk_dot64(w[t][j], a[j])), sc, acc[t]);
      }
    }
#pragma unroll
    for (int off = 1; off < LPR; off <<= 1)
#pragma unroll
      for (int t = 0; t < RPT; ++t) acc[t] += __shfl_xor_sync(kFull, acc[t], off);
    if (sub == 0)
#pragma unroll
      for (int t = 0; t < RPT; ++t)
        if (r[t] < k) out[r[t]] = has_bias ? acc[t] * act_scale + bias[r[t]] : acc[t] * act_scale;
  }
}

// Fallback for inputs with more than three chunks per lane: activations re-read from shared memory,
// chunk sums from xsum (the quantiser fills it for these ops).
__device__ __forceinline__ void chunk_rows_wide(const Op& op, const unsigned char* stage, int k, const int8_t* act,
                                                const int* xsum, float act_scale, float* out) {
  const int tid = threadIdx.x;
  const int lg = op.lpr_log;
  const int lpr = 1 << lg;
  const int rpi = kThreads >> lg;
  const int chunks = (op.in_n + 63) >> 6;
  const uint16_t* scales = reinterpret_cast<const uint16_t*>(stage + static_cast<size_t>(k) * op.row_bytes);
  const float* bias =
      reinterpret_cast<const float*>(stage + static_cast<size_t>(k) * op.row_bytes + round16(k * op.scale_stride * 2));
  const int sub = tid & (lpr - 1);
  for (int base = 0; base < k; base += rpi) {
    const int r = base + (tid >> lg);
    float acc = 0.0f;
    if (r < k) {
      const uint4* wrow = reinterpret_cast<const uint4*>(stage + static_cast<size_t>(r) * op.row_bytes);
      const uint16_t* srow = scales + r * op.scale_stride;
#pragma unroll 2
      for (int u = sub; u < chunks; u += lpr)
        acc = fmaf(static_cast<float>(chunk_dot_regs(wrow[u], load_act_chunk(act, xsum, u))), h2f(srow[u >> 1]), acc);
    }
    for (int off = 1; off < lpr; off <<= 1) acc += __shfl_xor_sync(kFull, acc, off);
    if (r < k && sub == 0) out[r] = op.has_bias ? acc * act_scale + bias[r] : acc * act_scale;
  }
}

__device__ __forceinline__ void chunk_rows(const Op& op, const unsigned char* stage, int k, const int8_t* act, const int* xsum,
                           float act_scale, float* out) {
  const int chunks = (op.in_n + 63) >> 6;
  const int kpl = (chunks + (1 << op.lpr_log) - 1) >> op.lpr_log;
  switch (kpl) {
    case 1: chunk_rows_kpl<1, 4>(op, stage, k, act, xsum, act_scale, out); break;
    case 2: chunk_rows_kpl<2, 4>(op, stage, k, act, xsum, act_scale, out); break;
    case 3: chunk_rows_kpl<3, 2>(op, stage, k, act, xsum, act_scale, out); break;
    default: chunk_rows_wide(op, stage, k, act, xsum, act_scale, out); break;
  }
}

// ---- top-k selection (radix select over order-preserving keys) ----------------------------------
struct TopkScratch {
  unsigned* hist;  // [kWarps * 256]
  int* misc;       // [16]
};

static __device__ int topk_digit(const TopkScratch& ts, const unsigned* keys, int n, int shift, unsigned& prefix,
                                 unsigned& mask, int& remaining) {
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
  prefix |= static_cast<unsigned>(ts.misc[8]) << shift;
  mask |= 255u << shift;
  remaining = ts.misc[9];
  __syncthreads();
  return 0;
}

// The K best of keys[0, n) by (key desc, id asc); ids[i] (or id_base + i when ids == nullptr) must
// increase with i among equal keys. Writes them sorted into out_key / out_id (K <= kMaxTopK).
static __device__ void topk_sorted(const unsigned* keys, const int* ids, int id_base, int n, int K, const TopkScratch& ts,
                                   unsigned* ck, int* ci, unsigned* out_key, int* out_id) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  unsigned prefix = 0u, mask = 0u;
  int remaining = K;
  for (int shift = 24; shift >= 0; shift -= 8) topk_digit(ts, keys, n, shift, prefix, mask, remaining);
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
static __device__ int draw_token(const unsigned* sorted_key, const int* sorted_id, int K, float* cdf, float* red,
                                 uint64_t key, uint64_t counter) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float top = key_value(sorted_key[0]);
  for (int c = tid; c < K; c += kThreads) cdf[c] = expf(key_value(sorted_key[c]) - top);
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

namespace ivb {
// true when chunk_rows reads the quantiser's chunk sums (more than three chunks per lane)
__host__ __device__ __forceinline__ bool op_needs_xsum(const Op& op) {
  const int chunks = (op.in_n + 63) >> 6;
  return ((chunks + (1 << op.lpr_log) - 1) >> op.lpr_log) > 3;
}
}  // namespace ivb
