// Persistent multi-layer decode kernel of libivonar_b200.so.
//
// One cooperative launch runs `steps` tokens: for every token the CTAs (one per SM) walk a phase
// program built on the host — per block: fused norm+quantise+GEMV entry projection, the recurrent
// step or latent attention, the out projection with residual add, the SwiGLU gate/up GEMV and the
// down GEMV with residual add — then the LM head and the sampler. Phases are separated by a bounded
// grid barrier; each CTA loads the first weight chunks of its next GEMV slice into registers before
// it waits, so the weight stream overlaps the barrier latency. This replaces the reference's 131-137
// launches per token and its 16-token CUDA graph (kernel_decoder.py:179-283, 683-735).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "ivb_common.h"
#include "ivb_cluster.cuh"

size_t ivb_sample_smem_bytes(int vocab);
size_t ivb_gemv_smem_bytes(int n);
int ivb_lpr_log(int in_features);

namespace ivb {


// floats of the recurrent constants copied out of the constants chunk: decay, theta, skip, conv w/b
__host__ __device__ __forceinline__ int ssm_const_floats(int nh, int S, int hd, int taps) {
  return 2 * nh * S + nh * hd * (2 + taps);
}
__device__ __forceinline__ void cp_async_f32(float* dst, const float* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

constexpr int kAttnPieces = 4;

// Copy src[0, n) (local shared memory, written before a __syncthreads) to dst[base, base + n) in every
// CTA of the cluster; the bytes complete on that CTA's mbarrier `bar` (the consumer arms it with the
// size of the whole fill and waits). Aligned slices go as one bulk shared-to-shared copy per CTA,
// issued by thread r for CTA r (the copy engine reads src; push_drain() waits for those reads before
// src is written again); other slices as one st.async per (word, rank).
__device__ __forceinline__ void push_async(float* dst, int base, const float* src, int n, int R, unsigned long long* bar) {
  if (((base | n) & 3) == 0) {
    if (static_cast<int>(threadIdx.x) < R && n > 0) {
      fence_proxy_async();  // the generic writes of src (ordered by the barrier) before the async-proxy read
      asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       map_rank(dst + base, threadIdx.x)),
                   "r"(smem_addr(src)), "r"(static_cast<unsigned>(n) * 4u), "r"(map_rank(bar, threadIdx.x))
                   : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
  } else {
    for (int idx = threadIdx.x; idx < n * R; idx += kThreads) {
      const int r = idx / n, i = idx - r * n;
      st_async_b32(map_rank(dst + base + i, r), __float_as_uint(src[i]), map_rank(bar, r));
    }
  }
}
// Every thread: wait until the bulk pushes this thread issued have read their source.
__device__ __forceinline__ void push_drain() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Bounded wait on an attention tile mbarrier; the verdict is uniform across the CTA.
__device__ __forceinline__ bool tile_wait(unsigned long long* bar, unsigned parity, unsigned long long timeout_ns) {
  const bool late = !mbar_wait_bounded(bar, parity, timeout_ns);
  return !__syncthreads_or(late);
}

struct TileBuf {
  int8_t* lat;      // [tile][lpad]
  float* lsc;       // [tile]
  uint16_t* kr;     // [tile][rpad]
};

__device__ __forceinline__ TileBuf tile_buf(unsigned char* base, const ClusterDims& D, int b) {
  const size_t one = round16(D.tile * D.lpad) + round16(D.tile * 4) + round16(D.tile * D.rpad * 2);
  unsigned char* t = base + b * one;
  TileBuf tb;
  tb.lat = reinterpret_cast<int8_t*>(t);
  tb.lsc = reinterpret_cast<float*>(t + round16(D.tile * D.lpad));
  tb.kr = reinterpret_cast<uint16_t*>(t + round16(D.tile * D.lpad) + round16(D.tile * 4));
  return tb;
}

// thread 0: bulk-copy cached positions [start, start + count) of head h into tile buffer b
__device__ __forceinline__ void tile_issue(const IvbLayerDesc& L, const ClusterDims& D, const TileBuf& tb, int h,
                                           int start, int count, unsigned long long* bar) {
  const unsigned lat = count * D.lpad, lsc = round16(count * 4), kr = count * D.rpad * 2;
  asm volatile("fence.proxy.async.global;" ::: "memory");
  fence_proxy_async();
  mbar_expect_tx(bar, lat + lsc + kr);
  bulk_copy(tb.lat, L.latent_q + static_cast<size_t>(start) * D.lpad, lat, bar);
  bulk_copy(tb.lsc, L.latent_scale + start, lsc, bar);
  bulk_copy(tb.kr, L.k_rope_cache + (static_cast<size_t>(h) * D.max_len + start) * D.rpad, kr, bar);
}

// Rows of all stages of a GEMV op with compile-time lane geometry; the lane's activation chunks are
// loaded once and stay in registers across the stages. Returns false when a stage wait ran out.
template <int LG, int KPL, int RPT, typename Tick>
__device__ __forceinline__ bool rows_ct(const ClusterParams& p, Stream& st, unsigned rank, const Op& op, int rows_c,
                                        const int8_t* act, float act_scale, float* rows_out, Tick& tick) {
  const int chunks = (op.in_n + 63) >> 6;
  const int row_bytes = op.row_bytes, sstride = op.scale_stride;
  const bool has_bias = op.has_bias != 0;
  const int n_row_chunks = op.n_chunks - op.has_const, crows = op.chunk_rows;
  ActChunk a[KPL];
  bool have[KPL];
  load_act_ct<LG, KPL>(act, chunks, a, have);
  bool ok = true;
  for (int c = 0; c < n_row_chunks; ++c) {
    const unsigned char* stage = stream_acquire(p, st);
    tick(2);
    if (stage == nullptr) {
      ok = false;
    } else {
      const int r0 = c * crows;
      rows_stage_ct<LG, KPL, RPT>(a, have, stage, max(0, min(crows, rows_c - r0)), row_bytes, sstride, has_bias, act_scale,
                                  rows_out + r0);
    }
    tick(3);
    stream_release(p, st, rank);
    tick(4);
  }
  return ok;
}

// rope table of an mla block (the entry op's layer description)
__device__ __forceinline__ const float* L_entry_rope(const IvbLayerDesc& L) { return L.rope; }

__global__ void __launch_bounds__(kThreads, 1) cluster_decode_kernel(const __grid_constant__ ClusterParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) unsigned long long full[kStages];
  __shared__ __align__(8) unsigned long long abar[2];
  __shared__ __align__(8) unsigned long long xbar[XB_COUNT];  // fills of the pushed buffers (transaction counts)
  __shared__ __align__(16) OpRec opbuf[2];  // the running op and the next one (descriptor + layer)
  __shared__ __align__(16) int rowsbuf[2][4];
  const unsigned rank = cluster_rank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const ClusterDims& D = p.d;
  const ClusterSmem& M = p.sm;
  const int R = D.R;
  float* xv = reinterpret_cast<float*>(smem + M.xv);
  int8_t* act = reinterpret_cast<int8_t*>(smem + M.act);
  int* xsum = reinterpret_cast<int*>(smem + M.xsum);
  float* resid = reinterpret_cast<float*>(smem + M.resid);
  float* loc = reinterpret_cast<float*>(smem + M.loc);
  float* red = reinterpret_cast<float*>(smem + M.red);
  float* xl = reinterpret_cast<float*>(smem + M.xl);
  float* stg = reinterpret_cast<float*>(smem + M.pub);  // this op's output slice before it is pushed
  unsigned char* U = smem + M.u;
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    mbar_init(&abar[0], 1);
    mbar_init(&abar[1], 1);
    for (int b = 0; b < XB_COUNT; ++b) mbar_init(&xbar[b], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  unsigned long long* coff = reinterpret_cast<unsigned long long*>(smem + M.ctab);
  unsigned* cbytes = reinterpret_cast<unsigned*>(coff + p.chunks_per_token);
  for (int c = tid; c < p.chunks_per_token; c += kThreads) {
    coff[c] = p.chunk_off[static_cast<size_t>(rank) * p.chunks_per_token + c];
    cbytes[c] = p.chunk_bytes[static_cast<size_t>(rank) * p.chunks_per_token + c];
  }
  float* rope_s = reinterpret_cast<float*>(smem + M.rope_row);
  float* seen_s = reinterpret_cast<float*>(smem + M.seen);  // bytes; float* for the 4-byte copies
  __syncthreads();
  cluster_sync();
  Stream st{full, smem + M.ring, M.stage_bytes, coff, cbytes, 0u, 0u, 0, 0};
  // op descriptors travel through a two-slot shared buffer: op k+1 is fetched while op k runs
  auto fetch_op = [&](int oi, int slot) {
    if (tid < static_cast<int>(sizeof(OpRec) / 16))
      cp_async_16(reinterpret_cast<unsigned char*>(&opbuf[slot]) + 16 * tid,
                  reinterpret_cast<const unsigned char*>(p.ops + oi) + 16 * tid);
    else if (tid == kThreads - 1)
      cp_async_f32(reinterpret_cast<float*>(&rowsbuf[slot][0]), reinterpret_cast<const float*>(p.op_rows + oi * R + rank));
    cp_async_commit();
  };
  fetch_op(0, 0);
  cp_async_wait_all();
  __syncthreads();
  unsigned opk = 0;  // ops run so far (selects the descriptor slot)
  if (tid == 0)
    for (int k = 0; k < kStages; ++k) stream_issue(p, st, rank);
  unsigned apar[2] = {0u, 0u};
  const int first_head = static_cast<int>(rank) * D.hpc;
  const int nh = max(0, min(D.heads - first_head, D.hpc));
  long long pos = ldcg_i64(p.position);
  long long tok = p.feed != nullptr ? ldcg_i64(p.feed) : ldcg_i64(p.token);
  uint64_t rkey = p.rng[0], rctr = p.rng[1];
  const float inv_t = 1.0f / __ldcg(p.sampling);
  const float pen = __ldcg(p.sampling + 1), ipen = __ldcg(p.sampling + 2);
  const bool sampling = (p.flags & IVB_RUN_SAMPLE) != 0;
  int K = 1;
  {
    const long long kreq = ldcg_i64(p.top_k);
    const int cap = min(min(D.max_top_k, D.vocab), kMaxTopK);
    K = static_cast<int>(kreq < 1 ? 1 : (kreq > cap ? cap : kreq));
  }
  bool alive = true;
  // Ops hand their outputs to the next op through pushed buffers: the consumer arms the buffer's
  // mbarrier with the bytes of the whole fill (arrive + expect_tx) and waits (bounded); the
  // producers' st.async stores complete those bytes. No cluster barrier per op: a CTA starts an op as
  // soon as its input has landed. A CTA is never more than one op ahead of another (every op needs
  // every CTA's output of the previous one), and every op reads its input buffer before it pushes, so
  // a fill never overwrites a buffer that is still being read.
  unsigned xph[XB_COUNT] = {0u, 0u, 0u, 0u};
  auto wait_fill = [&](int b, unsigned bytes) -> bool {
    if (tid == 0) mbar_expect_tx(&xbar[b], bytes);
    const bool late = !mbar_wait_bounded(&xbar[b], xph[b], p.timeout_ns);
    xph[b] ^= 1u;
    return !__syncthreads_or(late);
  };
  auto fail_here = [&](unsigned code) {
    if (tid == 0) atomicCAS(p.error, 0u, code);
  };
  bool resid_pending = false;  // the last op of the previous token pushed the residual without a head
  for (int step = 0; step < p.steps && alive; ++step) {
    if (step > 0 && p.feed != nullptr) tok = ldcg_i64(p.feed + step);
    if (pos < 0 || pos >= D.max_len || tok < 0 || tok >= D.vocab) {
      // every CTA sees the same values: stop together
      if (rank == 0 && tid == 0) atomicCAS(p.error, 0u, static_cast<unsigned>(pos >= D.max_len ? IVB_ECAPACITY : IVB_EINVAL));
      break;
    }
    const bool head = head_needed(p, step);
    const bool tracing = p.trace != nullptr && step == p.trace_step;
    if (resid_pending) {
      resid_pending = false;
      if (!wait_fill(XB_RESID, static_cast<unsigned>(D.hidden) * 4u)) {
        fail_here(IVB_ETIMEOUT);
        break;
      }
    }
    // embedding of the token -> residual replica (every CTA computes the whole row)
    {
      const uint8_t* erow = p.head.packed + static_cast<size_t>(tok) * p.head.row_bytes;
      const uint16_t* srow = p.head.scales + static_cast<size_t>(tok) * p.head.scale_stride;
      for (int i = tid; i < D.hidden; i += kThreads)
        resid[i] = static_cast<float>(((__ldg(erow + (i >> 2)) >> ((i & 3) << 1)) & 3) - 1) * h2f(__ldg(srow + (i >> 7)));
    }
    __syncthreads();
    const int n_run = head ? p.n_ops : p.n_ops - 1;  // the head is the last op of the program
    for (int oi = 0; oi < n_run && alive; ++oi) {
      const Op& op = opbuf[opk & 1].op;  // fields are read from shared memory where used
      const IvbLayerDesc& lay = opbuf[opk & 1].layer;
      const int rows_c = rowsbuf[opk & 1][0];
      fetch_op(oi + 1 < n_run ? oi + 1 : 0, (opk + 1) & 1);  // the op after this one (op 0 of the next token)
      unsigned long long* marks = tracing ? p.trace + (static_cast<size_t>(oi) * R + rank) * 8 : nullptr;
      mark(marks, 0);
      // the input of this op (resid, xv or xl) was pushed into this CTA by every producer of the
      // previous op before the cluster barrier
      // tracing: slots 1..6 sum the SM cycles spent in six parts of the op (thread 0's view)
      long long prof[6] = {0, 0, 0, 0, 0, 0};
      long long prof_t = marks != nullptr ? clock64() : 0;
      auto tick = [&](int part) {
        if (marks != nullptr) {
          const long long now = clock64();
          prof[part] += now - prof_t;
          prof_t = now;
        }
      };
      const int lo = min(op.rows_total, static_cast<int>(rank) * op.rows_per);
      bool ok = true;
      if (op.in_buf >= 0 && !wait_fill(op.in_buf, static_cast<unsigned>(op.in_bytes))) {
        fail_here(IVB_ETIMEOUT);
        alive = false;
        break;
      }
      if (op.kind == OP_ATTN) {
        // ---------------- latent attention over the compressed cache ----------------
        const IvbLayerDesc& L = lay;
        const unsigned char* cst = stream_acquire(p, st);
        if (cst == nullptr) ok = false;
        float* qlat_f = reinterpret_cast<float*>(U);  // [latent] quantiser scratch
        int8_t* qlc = reinterpret_cast<int8_t*>(U + round16(((D.latent + 63) / 64 * 64) * 4));
        float* qa = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(qlc) + round16((D.latent + 63) / 64 * 64));
        float* qr = qa + D.latent;
        float* krc = qr + D.rope;
        float* qn = krc + D.rope;
        float* sc = qn + D.nope;
        float* part = sc + D.tile + 4;
        unsigned char* tiles = reinterpret_cast<unsigned char*>(part + kWarps * D.latent);
        tiles += (16 - (reinterpret_cast<uintptr_t>(tiles) & 15)) & 15;
        const float a_cur = quantize_block(xl, D.latent, nullptr, 0.0f, 0.0f, D.act_eps, qlc, false, nullptr, red);
        if (rank == 0) {
          for (int j = tid; j < D.latent; j += kThreads) L.latent_q[static_cast<size_t>(pos) * D.lpad + j] = qlc[j];
          if (tid == 0) L.latent_scale[pos] = a_cur;
        }
        const int P = static_cast<int>(pos);
        const int n_tiles = P == 0 ? 1 : (P + D.tile - 1) / D.tile;
        tick(0);
        for (int hl = 0; hl < nh && ok; ++hl) {
          const int h = first_head + hl;
          const float* qh = loc + hl * D.head_dim;
          const float* kh = loc + nh * D.head_dim + hl * D.rope;
          const float scl = L.attn_scale;
          for (int jr = tid; jr < D.rope / 2; jr += kThreads) {
            const float cs = rope_s[2 * jr], sn = rope_s[2 * jr + 1];  // prefetched by the entry op
            const float q0 = qh[D.nope + 2 * jr], q1 = qh[D.nope + 2 * jr + 1];
            const float k0 = kh[2 * jr], k1 = kh[2 * jr + 1];
            qr[2 * jr] = (q0 * cs - q1 * sn) * scl;
            qr[2 * jr + 1] = (q0 * sn + q1 * cs) * scl;
            const float kr0 = k0 * cs - k1 * sn, kr1 = k0 * sn + k1 * cs;
            krc[2 * jr] = kr0;
            krc[2 * jr + 1] = kr1;
            uint16_t* kc = L.k_rope_cache + (static_cast<size_t>(h) * D.max_len + P) * D.rpad;
            kc[2 * jr] = f2h(kr0);
            kc[2 * jr + 1] = f2h(kr1);
          }
          for (int e = tid; e < D.nope; e += kThreads) qn[e] = qh[e] * scl;
          // first tile of this head
          if (tid == 0 && P > 0) tile_issue(L, D, tile_buf(tiles, D, 0), h, 0, min(P, D.tile), &abar[0]);
          __syncthreads();
          // absorbed query qa[j] = sum_e qn[e] * W_knope[h][e][j] (weights in the constants chunk)
          const unsigned char* wkn = cst + op.c_wkn + static_cast<size_t>(hl) * D.nope * D.rb_lat;
          const uint16_t* skn = reinterpret_cast<const uint16_t*>(cst + op.c_skn) + hl * D.nope * D.ss_lat;
          const int words = (D.latent + 15) >> 4;  // 16-input words of a latent row
          if ((words & (words - 1)) == 0) {
            // thread: word wd of e-group eg; the e-groups of a warp meet by shuffles, the warps in `part`
            const int wd = tid & (words - 1), eg = tid / words, n_eg = kThreads / words;
            float acc[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = 0.0f;
            for (int e = eg; e < D.nope; e += n_eg) {
              const unsigned w = *reinterpret_cast<const unsigned*>(wkn + e * D.rb_lat + wd * 4);
              const float sc_e = h2f(skn[e * D.ss_lat + (wd >> 3)]), q_e = qn[e];
              float cm1[16];
              word_codes_m1(w, cm1);
#pragma unroll
              for (int i = 0; i < 16; ++i) acc[i] = fmaf(q_e, cm1[i] * sc_e, acc[i]);
            }
            for (int off = words; off < 32; off <<= 1)
#pragma unroll
              for (int i = 0; i < 16; ++i) acc[i] += __shfl_xor_sync(kFull, acc[i], off);
            if (lane < words)
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (wd * 16 + i < D.latent) part[warp * D.latent + wd * 16 + i] = acc[i];
            __syncthreads();
            for (int j = tid; j < D.latent; j += kThreads) {
              float v = part[j];
#pragma unroll
              for (int w2 = 1; w2 < kWarps; ++w2) v += part[w2 * D.latent + j];
              qa[j] = v;
            }
          } else {
            for (int j = tid; j < D.latent; j += kThreads) {
              float acc = 0.0f;
              for (int e = 0; e < D.nope; ++e)
                acc = fmaf(qn[e], code_value(wkn + e * D.rb_lat, j) * h2f(skn[e * D.ss_lat + (j >> 7)]), acc);
              qa[j] = acc;
            }
          }
          float qb = 0.0f;
          if (L.k_nope_up.bias != nullptr) {
            const float* bkn = reinterpret_cast<const float*>(cst + op.c_bkn) + hl * D.nope;
            float pp = 0.0f;
            for (int e = tid; e < D.nope; e += kThreads) pp = fmaf(qn[e], bkn[e], pp);
            qb = block_sum(pp, red);
          } else {
            __syncthreads();
          }
          // Tiles of cached positions (plus the current one, last): scores with 8 lanes per position
          // (lane `sub` owns latent pieces p * 128 + sub * 16 .. + 16, the absorbed query slice kept in
          // registers), an online softmax, and the weighted latent sum u with one warp per position
          // group (lane owns latent lane * 8 + 256 * p2 .. + 8).
          tick(1);
          const int sub = tid & 7, grp = tid >> 3;
          float qa_r[kAttnPieces][16];
#pragma unroll
          for (int pc = 0; pc < kAttnPieces; ++pc)
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int j = pc * 128 + sub * 16 + i;
              qa_r[pc][i] = j < D.latent ? qa[j] : 0.0f;
            }
          float u[kAttnPieces / 2 > 0 ? kAttnPieces / 2 : 1][8];
#pragma unroll
          for (int pc = 0; pc < (kAttnPieces / 2 > 0 ? kAttnPieces / 2 : 1); ++pc)
#pragma unroll
            for (int i = 0; i < 8; ++i) u[pc][i] = 0.0f;
          float m_run = -INFINITY, l_run = 0.0f;
          for (int ti = 0; ti < n_tiles; ++ti) {
            tick(5);
            const int start = ti * D.tile;
            const int count = max(0, min(D.tile, P - start));
            const bool last = ti == n_tiles - 1;
            const TileBuf tb = tile_buf(tiles, D, ti & 1);
            if (tid == 0 && ti + 1 < n_tiles)
              tile_issue(L, D, tile_buf(tiles, D, (ti + 1) & 1), h, start + D.tile, min(D.tile, P - start - D.tile),
                         &abar[(ti + 1) & 1]);
            if (count > 0) {
              if (!tile_wait(&abar[ti & 1], apar[ti & 1], p.timeout_ns)) {
                ok = false;
                break;
              }
              apar[ti & 1] ^= 1u;
            }
            tick(4);
            const int npos = count + (last ? 1 : 0);
            for (int k = grp; k - grp < npos; k += kThreads / 8) {
              const bool valid = k < npos;
              const bool cur = k == count;
              const int8_t* ql = cur ? qlc : tb.lat + (valid ? k : 0) * D.lpad;
              float dot0 = 0.0f, dot1 = 0.0f;
#pragma unroll
              for (int pc = 0; pc < kAttnPieces; ++pc) {
                const int j0 = pc * 128 + sub * 16;
                if (valid && j0 < D.latent) {
                  const uint4 w = *reinterpret_cast<const uint4*>(ql + j0);
                  float f[16];
                  bytes_to_f32(w.x, f);
                  bytes_to_f32(w.y, f + 4);
                  bytes_to_f32(w.z, f + 8);
                  bytes_to_f32(w.w, f + 12);
#pragma unroll
                  for (int i = 0; i < 16; i += 2) {
                    dot0 = fmaf(qa_r[pc][i], f[i], dot0);
                    dot1 = fmaf(qa_r[pc][i + 1], f[i + 1], dot1);
                  }
                }
              }
              float rp = 0.0f;
              if (valid)
                for (int r = sub; r < D.rope; r += 8) rp = fmaf(qr[r], cur ? krc[r] : h2f(tb.kr[k * D.rpad + r]), rp);
              const float at = valid ? (cur ? a_cur : tb.lsc[k]) : 0.0f;
              float total = fmaf(at, dot0 + dot1, rp);
              total += __shfl_xor_sync(kFull, total, 4);
              total += __shfl_xor_sync(kFull, total, 2);
              total += __shfl_xor_sync(kFull, total, 1);
              if (valid && sub == 0) sc[k] = total + qb;
            }
            __syncthreads();
            tick(2);
            float mx = -INFINITY;
            for (int k = tid; k < npos; k += kThreads) mx = fmaxf(mx, sc[k]);
            mx = block_max(mx, red);
            const float m_new = fmaxf(m_run, mx);
            const float corr = m_run == -INFINITY ? 0.0f : expf(m_run - m_new);
            float ls = 0.0f;
            for (int k = tid; k < npos; k += kThreads) {
              const float e = expf(sc[k] - m_new);
              sc[k] = e * (k == count ? a_cur : tb.lsc[k]);  // softmax weight times the latent scale
              ls += e;
            }
            ls = block_sum(ls, red);
            l_run = l_run * corr + ls;
#pragma unroll
            for (int pc = 0; pc < (kAttnPieces / 2 > 0 ? kAttnPieces / 2 : 1); ++pc)
#pragma unroll
              for (int i = 0; i < 8; ++i) u[pc][i] *= corr;
            for (int k = warp; k < npos; k += kWarps) {
              const int8_t* ql = k == count ? qlc : tb.lat + k * D.lpad;
              const float ea = sc[k];
#pragma unroll
              for (int pc = 0; pc < (kAttnPieces / 2 > 0 ? kAttnPieces / 2 : 1); ++pc) {
                const int j0 = pc * 256 + lane * 8;
                if (j0 < D.latent) {
                  const uint2 w = *reinterpret_cast<const uint2*>(ql + j0);
                  float f[8];
                  bytes_to_f32(w.x, f);
                  bytes_to_f32(w.y, f + 4);
#pragma unroll
                  for (int i = 0; i < 8; ++i) u[pc][i] = fmaf(ea, f[i], u[pc][i]);
                }
              }
            }
            m_run = m_new;
            __syncthreads();
          }
          if (!ok) break;
          tick(5);
#pragma unroll
          for (int pc = 0; pc < (kAttnPieces / 2 > 0 ? kAttnPieces / 2 : 1); ++pc) {
            const int j0 = pc * 256 + lane * 8;
#pragma unroll
            for (int i = 0; i < 8; ++i)
              if (j0 + i < D.latent) part[warp * D.latent + j0 + i] = u[pc][i];
          }
          __syncthreads();
          for (int j = tid; j < D.latent; j += kThreads) {
            float v = part[j];
#pragma unroll
            for (int w = 1; w < kWarps; ++w) v += part[w * D.latent + j];
            qlat_f[j] = v;
          }
          __syncthreads();
          // out_h[e] = W_v[h][e] . u / l + b_v
          const unsigned char* wv = cst + op.c_wv + static_cast<size_t>(hl) * D.head_dim * D.rb_lat;
          const uint16_t* sv = reinterpret_cast<const uint16_t*>(cst + op.c_sv) + hl * D.head_dim * D.ss_lat;
          const float* bv = reinterpret_cast<const float*>(cst + op.c_bv) + hl * D.head_dim;
          const float inv_l = 1.0f / l_run;
          if ((words & (words - 1)) == 0) {
            // lanes of a row own its 16-input words (the u slice in registers); rows step by kThreads/words
            const int wd = tid & (words - 1);
            float uj[16], cm1[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) uj[i] = wd * 16 + i < D.latent ? qlat_f[wd * 16 + i] : 0.0f;
            for (int e0 = 0; e0 < D.head_dim; e0 += kThreads / words) {
              const int e = e0 + tid / words;
              float acc = 0.0f;
              if (e < D.head_dim) {
                const unsigned w = *reinterpret_cast<const unsigned*>(wv + e * D.rb_lat + wd * 4);
                const float sc_e = h2f(sv[e * D.ss_lat + (wd >> 3)]);
                word_codes_m1(w, cm1);
#pragma unroll
                for (int i = 0; i < 16; ++i) acc = fmaf(cm1[i] * sc_e, uj[i], acc);
              }
              for (int off = 1; off < words; off <<= 1) acc += __shfl_xor_sync(kFull, acc, off);
              if (e < D.head_dim && wd == 0) {
                float o = acc * inv_l;
                if (L.v_up.bias != nullptr) o += bv[e];
                stg[hl * D.head_dim + e] = o;
              }
            }
          } else {
          int tpr = kThreads / D.head_dim;
          if (tpr > 32) tpr = 32;
          int tpr_log = 0;
          while ((2 << tpr_log) <= tpr) ++tpr_log;
          tpr = 1 << tpr_log;
          for (int base = 0; base < D.head_dim; base += kThreads >> tpr_log) {
            const int e = base + (tid >> tpr_log);
            const int pid = tid & (tpr - 1);
            float acc = 0.0f;
            if (e < D.head_dim) {
              const unsigned char* row = wv + e * D.rb_lat;
              const int span = (D.latent + tpr - 1) / tpr;
              const int j0 = pid * span, j1 = min(D.latent, j0 + span);
              for (int j = j0; j < j1; ++j) acc = fmaf(code_value(row, j) * h2f(sv[e * D.ss_lat + (j >> 7)]), qlat_f[j], acc);
            }
            for (int off = 1; off < tpr; off <<= 1) acc += __shfl_xor_sync(kFull, acc, off);
            if (e < D.head_dim && pid == 0) {
              float o = acc * inv_l;
              if (L.v_up.bias != nullptr) o += bv[e];
              stg[hl * D.head_dim + e] = o;
            }
          }
          }
          __syncthreads();
          tick(3);
        }
        if (ok) push_async(xv, first_head * D.head_dim, stg, nh * D.head_dim, R, &xbar[XB_VEC]);  // stg written before the head loop's last sync
        asm volatile("fence.proxy.async.global;" ::: "memory");
        if (!ok) fail_here(IVB_ETIMEOUT);
        stream_release(p, st, rank);
      } else {
        // ---------------- GEMV ops ----------------
        const unsigned char* cst = nullptr;
        float act_scale = 0.0f;
        float* ssmc = reinterpret_cast<float*>(U);
        const int S = D.state_dim, hd = D.head_dim, taps = D.taps;
        if (op.kind == OP_ENTRY_MLA) {
          // the rope row of this position, for the attention op that follows
          const float* rrow = L_entry_rope(lay) + static_cast<size_t>(pos) * D.rope;
          for (int i = tid; i < D.rope; i += kThreads) cp_async_f32(rope_s + i, rrow + i);
          cp_async_commit();
        } else if (op.kind == OP_HEAD && sampling && ((lo | rows_c) & 3) == 0) {
          // the repetition flags of my vocabulary slice, for the local top-k
          const float* src = reinterpret_cast<const float*>(p.seen + lo);
          for (int i = tid; i < rows_c / 4; i += kThreads) cp_async_f32(seen_s + i, src + i);
          cp_async_commit();
        }
        if (op.kind == OP_ENTRY_MAMBA && nh > 0) {
          // the recurrent state of my heads streams into shared memory while the rows are computed
          const IvbLayerDesc& L = lay;
          const int nhs = nh * S, channels = nh * hd;
          float* dst = ssmc + ssm_const_floats(nh, S, hd, taps) + 5 * nhs + channels + max(kThreads, channels);
          const float* src[3] = {L.ssm_state + static_cast<size_t>(first_head) * S * hd * 2,
                                 L.prev_force + static_cast<size_t>(first_head) * S * hd,
                                 L.conv_state + static_cast<size_t>(first_head) * hd * (taps - 1)};
          const int len[3] = {2 * nhs * hd, nhs * hd, channels * (taps - 1)};
          for (int a2 = 0; a2 < 3; ++a2) {
            for (int i = tid; i < len[a2]; i += kThreads) cp_async_f32(dst + i, src[a2] + i);
            dst += len[a2];
          }
          cp_async_commit();
        }
        if (op.has_const) {
          cst = stream_acquire(p, st);
          if (cst == nullptr) ok = false;
        }
        tick(0);
        // quantiser input: the residual replica (entry, gate/up, head) or the pushed vector (out, down)
        const bool from_resid =
            op.kind == OP_ENTRY_MAMBA || op.kind == OP_ENTRY_MLA || op.kind == OP_GATE_UP || op.kind == OP_HEAD;
        const float* norm_w = (op.has_norm && cst != nullptr) ? reinterpret_cast<const float*>(cst + op.c_norm) : nullptr;
        act_scale = quantize_block(from_resid ? resid : xv, op.in_n, norm_w, op.norm_eps, D.clip, D.act_eps, act, true,
                                   op_needs_xsum(op) ? xsum : nullptr, red);
        tick(1);
        // SSM constants leave the stage before it is recycled
        if (op.kind == OP_ENTRY_MAMBA && cst != nullptr) {
          const float* src[5] = {reinterpret_cast<const float*>(cst + op.c_decay), reinterpret_cast<const float*>(cst + op.c_theta),
                                 reinterpret_cast<const float*>(cst + op.c_skip), reinterpret_cast<const float*>(cst + op.c_convw),
                                 reinterpret_cast<const float*>(cst + op.c_convb)};
          const int len[5] = {nh * S, nh * S, nh * hd, nh * hd * taps, nh * hd};
          int off = 0;
          for (int a = 0; a < 5; ++a) {
            for (int i = tid; i < len[a]; i += kThreads) ssmc[off + i] = src[a][i];
            off += len[a];
          }
        }
        if (op.has_const) stream_release(p, st, rank);
        // rows of this CTA, chunk by chunk
        float* rows_out = loc;
        const int n_row_chunks = op.n_chunks - op.has_const;
        const int kpl = (((op.in_n + 63) >> 6) + (1 << op.lpr_log) - 1) >> op.lpr_log;
        const int geo = op.lpr_log * 8 + kpl;
        bool done_ct = true;
        if (geo == 3 * 8 + 2) ok &= rows_ct<3, 2, 4>(p, st, rank, op, rows_c, act, act_scale, rows_out, tick);
        else if (geo == 4 * 8 + 3) ok &= rows_ct<4, 3, 3>(p, st, rank, op, rows_c, act, act_scale, rows_out, tick);
        else if (geo == 5 * 8 + 2) ok &= rows_ct<5, 2, 4>(p, st, rank, op, rows_c, act, act_scale, rows_out, tick);
        else if (geo == 5 * 8 + 3) ok &= rows_ct<5, 3, 2>(p, st, rank, op, rows_c, act, act_scale, rows_out, tick);
        else done_ct = false;
        for (int c = 0; c < (done_ct ? 0 : n_row_chunks); ++c) {
          const unsigned char* stage = stream_acquire(p, st);
          tick(2);
          if (stage == nullptr) {
            ok = false;
          } else {
            const int r0 = c * op.chunk_rows;
            const int k = max(0, min(op.chunk_rows, rows_c - r0));
            chunk_rows(op, stage, k, act, xsum, act_scale, rows_out + r0);
          }
          tick(3);
          stream_release(p, st, rank);
          tick(4);
        }
        // epilogues
        if (op.kind == OP_OUT || op.kind == OP_DOWN) {
          for (int r = tid; r < rows_c; r += kThreads) stg[r] = resid[lo + r] + rows_out[r];
          __syncthreads();
          push_async(resid, lo, stg, rows_c, R, &xbar[XB_RESID]);
        } else if (op.kind == OP_GATE_UP) {
          for (int m = tid; m < rows_c / 2; m += kThreads) stg[m] = silu_f(rows_out[2 * m]) * rows_out[2 * m + 1];
          __syncthreads();
          push_async(xv, lo / 2, stg, rows_c / 2, R, &xbar[XB_VEC]);
        } else if (op.kind == OP_ENTRY_MLA) {
          const int lat0 = nh * (D.head_dim + D.rope);
          const int l0 = static_cast<int>(rank) * op.push_per;  // first latent row of this CTA
          for (int r = tid; r < rows_c - lat0; r += kThreads) stg[r] = rows_out[lat0 + r];
          __syncthreads();
          push_async(xl, l0, stg, rows_c - lat0, R, &xbar[XB_LATENT]);
        } else if (op.kind == OP_HEAD) {
          for (int r = tid; r < rows_c; r += kThreads) p.logits[lo + r] = rows_out[r];
        } else if (op.kind == OP_ENTRY_MAMBA && nh > 0) {
          // recurrent step for the channels of my heads; rows_out = per head [value hd | gate hd | bc_dt 3S]
          const IvbLayerDesc& L = lay;
          const float* decay = ssmc;
          const float* theta = decay + nh * S;
          const float* skip = theta + nh * S;
          const float* convw = skip + nh * hd;
          const float* convb = convw + nh * hd * taps;
          const int channels = nh * hd, nhs = nh * S;
          float* coef = ssmc + ssm_const_floats(nh, S, hd, taps);  // [5][nh*S]: b, c, half_dt, a_re, a_im
          float* vals = coef + 5 * nhs;                            // [channels] conv + SiLU values
          float* cpart = vals + channels;                          // [max(kThreads, channels)] partial readouts
          const float* s_state = cpart + max(kThreads, channels);  // prefetched [nh][S][hd][2]
          const float* s_prev = s_state + 2 * nhs * hd;             // [nh][S][hd]
          const float* s_conv = s_prev + nhs * hd;                  // [channels][taps - 1]
          cp_async_wait_all();
          __syncthreads();
          for (int t = tid; t < nhs; t += kThreads) {
            const int hl = t / S, s2 = t - hl * S;
            const float* bcdt = rows_out + hl * (2 * hd + 3 * S) + 2 * hd;
            const float half_dt = D.half_dt_min + sigmoid_f(bcdt[2 * S + s2]) * D.half_dt_range;
            const float mag = expf(2.0f * half_dt * decay[t]);
            float sn, cs;
            sincosf(2.0f * half_dt * theta[t], &sn, &cs);
            coef[t] = tanhf(bcdt[s2]);
            coef[nhs + t] = tanhf(bcdt[S + s2]);
            coef[2 * nhs + t] = half_dt;
            coef[3 * nhs + t] = mag * cs;
            coef[4 * nhs + t] = mag * sn;
          }
          for (int cl = tid; cl < channels; cl += kThreads) {
            const int hl = cl / hd, dd = cl - hl * hd;
            const float* win = s_conv + cl * (taps - 1);
            float* gwin = L.conv_state + static_cast<size_t>(first_head * hd + cl) * (taps - 1);
            const float incoming = rows_out[hl * (2 * hd + 3 * S) + dd];
            float conv = convb[cl];
            for (int k2 = 0; k2 < taps - 1; ++k2) conv = fmaf(convw[cl * taps + k2], win[k2], conv);
            conv = fmaf(convw[cl * taps + taps - 1], incoming, conv);
            for (int k2 = 0; k2 + 1 < taps - 1; ++k2) gwin[k2] = win[k2 + 1];
            if (taps > 1) gwin[taps - 2] = incoming;
            vals[cl] = silu_f(conv);
          }
          __syncthreads();
          // thread (group g, channel cl) advances states g*spt .. of channel cl; lanes run along the
          // channels so the state loads and stores are contiguous
          const int groups = max(1, min(S, kThreads / channels));
          const int spt = (S + groups - 1) / groups;
          for (int it = tid; it < groups * channels; it += kThreads) {
            const int g = it / channels, cl = it - g * channels;
            const int hl = cl / hd, dd = cl - hl * hd;
            const float value = vals[cl];
            float contrib = 0.0f;
            for (int s2 = g * spt; s2 < min(S, (g + 1) * spt); ++s2) {
              const int t = hl * S + s2;
              const int li = t * hd + dd;  // local state index
              const size_t gi = static_cast<size_t>(first_head * S + t) * hd + dd;
              const float b = coef[t], cc = coef[nhs + t], half_dt = coef[2 * nhs + t];
              const float ar = coef[3 * nhs + t], ai = coef[4 * nhs + t];
              const float prev = s_prev[li];
              const float sr = s_state[2 * li], si = s_state[2 * li + 1];
              const float force = b * value;
              const float dr = (force + ar * prev) * half_dt;
              const float di = (ai * prev) * half_dt;
              const float nr = sr * ar - si * ai + dr;
              const float ni = sr * ai + si * ar + di;
              reinterpret_cast<float2*>(L.ssm_state)[gi] = make_float2(nr, ni);
              L.prev_force[gi] = force;
              contrib = fmaf(cc, nr, contrib);
            }
            cpart[it] = contrib;
          }
          __syncthreads();
          for (int cl = tid; cl < channels; cl += kThreads) {
            const int hl = cl / hd, dd = cl - hl * hd;
            float contrib = 0.0f;
            for (int g = 0; g < groups; ++g) contrib += cpart[g * channels + cl];
            const float y = (contrib + skip[cl] * vals[cl]) * sigmoid_f(rows_out[hl * (2 * hd + 3 * S) + hd + dd]);
            stg[cl] = y;
          }
          __syncthreads();
          push_async(xv, first_head * hd, stg, channels, R, &xbar[XB_VEC]);
        }
        if (!ok) fail_here(IVB_ETIMEOUT);
        // the head ends the token: local top-k of my vocabulary slice for the sampler
        if (op.kind == OP_HEAD && sampling) {
          // head scratch at U: keys [rows_per] | ck, ci, out keys, out ids [kc] | histogram | misc;
          // the merge arrays that the other CTAs push into start at U + M.cand (disjoint)
          unsigned* keys = reinterpret_cast<unsigned*>(U);
          unsigned* ck = keys + op.rows_per;
          int* ci = reinterpret_cast<int*>(ck + p.kc);
          unsigned* ok_key = reinterpret_cast<unsigned*>(ci + p.kc);
          int* ok_id = reinterpret_cast<int*>(ok_key + p.kc);
          TopkScratch ts{reinterpret_cast<unsigned*>(ok_id + p.kc), reinterpret_cast<int*>(ok_id + p.kc) + kWarps * 256};
          cp_async_wait_all();
          __syncthreads();
          const uint8_t* seen_b = reinterpret_cast<const uint8_t*>(seen_s);
          const bool pref = ((lo | rows_c) & 3) == 0;
          for (int r = tid; r < rows_c; r += kThreads)
            keys[r] = score_key(rows_out[r], pref ? seen_b[r] : __ldcg(p.seen + lo + r), inv_t, pen, ipen);
          __syncthreads();
          const int kl = min(K, rows_c);
          if (kl > 0) topk_sorted(keys, nullptr, lo, rows_c, kl, ts, ck, ci, ok_key, ok_id);
          __syncthreads();
          // my candidates go to offset sum_{r < rank} min(K, rows of r) of every CTA's merge arrays
          int base = 0;
          for (int r = 0; r < static_cast<int>(rank); ++r)
            base += min(K, max(0, min(op.rows_total - r * op.rows_per, op.rows_per)));
          unsigned* mk = reinterpret_cast<unsigned*>(U + M.cand);
          int* mi = reinterpret_cast<int*>(mk + R * p.kc);
          for (int idx = tid; idx < kl * R; idx += kThreads) {
            const int r = idx / kl, c = idx - r * kl;
            const unsigned bar = map_rank(&xbar[XB_CAND], r);
            st_async_b32(map_rank(mk + base + c, r), ok_key[c], bar);
            st_async_b32(map_rank(mi + base + c, r), static_cast<unsigned>(ok_id[c]), bar);
          }
        }
      }
      tick(5);
      if (marks != nullptr && tid == 0)
        for (int k = 0; k < 6; ++k) marks[1 + k] = static_cast<unsigned long long>(prof[k]);
      mark(marks, 7);
      cp_async_wait_all();  // the next descriptor has landed
      push_drain();         // the staging slice has been read by this op's pushes
      ++opk;
      __syncthreads();      // local buffers (rows, codes, staging) are reused by the next op
      if (!ok) {
        alive = false;
        break;
      }
    }
    if (!alive) break;
    if (!head) resid_pending = true;
    if (sampling) {
      // every CTA merges the cluster's candidates (pushed into its merge arrays) and draws the same token
      const int kc = p.kc;
      const Op& hop = opbuf[(opk + 1) & 1].op;  // the head op just run (the slot before the current one)
      unsigned* mk = reinterpret_cast<unsigned*>(U + M.cand);
      int* mi = reinterpret_cast<int*>(mk + R * kc);
      unsigned* ck = reinterpret_cast<unsigned*>(U);
      int* ci = reinterpret_cast<int*>(ck + kc);
      unsigned* sk = reinterpret_cast<unsigned*>(ci + kc);
      int* si = reinterpret_cast<int*>(sk + kc);
      float* cdf = reinterpret_cast<float*>(si + kc);
      TopkScratch ts{reinterpret_cast<unsigned*>(cdf + kc), reinterpret_cast<int*>(cdf + kc) + kWarps * 256};
      int n = 0;
      for (int r = 0; r < R; ++r) n += min(K, max(0, min(hop.rows_total - r * hop.rows_per, hop.rows_per)));
      if (!wait_fill(XB_CAND, static_cast<unsigned>(n) * 8u)) {
        fail_here(IVB_ETIMEOUT);
        break;
      }
      const int kk = min(K, n);
      topk_sorted(mk, mi, 0, n, kk, ts, ck, ci, sk, si);
      const int chosen = draw_token(sk, si, kk, cdf, red, rkey, rctr);
      ++rctr;
      tok = chosen;
      if (tid == 0) {
        const int per = (D.vocab + R - 1) / R;
        if (chosen / per == static_cast<int>(rank)) p.seen[chosen] = 1;
        if (rank == 0) {
          p.token[0] = chosen;
          p.rng[1] = rctr;
          if (p.history != nullptr && step < p.history_len) p.history[step] = chosen;
        }
      }
    }
    ++pos;
    if (rank == 0 && tid == 0) p.position[0] = pos;
  }
  // let every in-flight copy land before the CTA's shared memory goes away: a residual fill nobody
  // consumed (the run stopped after a step without a head), the descriptor prefetch, the ring
  if (resid_pending) wait_fill(XB_RESID, static_cast<unsigned>(D.hidden) * 4u);
  cp_async_wait_all();
  push_drain();
  if (tid == 0) {
    while (st.consumed < st.issued) {
      if (!mbar_wait_bounded(st.full + st.consumed % kStages, (st.consumed / kStages) & 1u, p.timeout_ns)) break;
      ++st.consumed;
    }
  }
  __syncthreads();
  cluster_sync();
}

}  // namespace ivb

// ------------------------------------------------------------------------------------------------
// host plan: per-CTA weight streams, op program, shared-memory map
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
  ivb::ClusterDims d;
  ivb::ClusterSmem sm;
  std::vector<ivb::Op> ops;
  std::vector<ivb::OpRec> recs;  // device op records, kept alive until the upload completes
  std::vector<int32_t> op_rows;
  std::vector<unsigned long long> chunk_off;
  std::vector<unsigned> chunk_bytes;
  std::vector<CopyOp> copies;
  int32_t R, cpt, head_first, kc;
  size_t stream_bytes, smem;
  size_t off_stream, off_ops, off_op_rows, off_chunk_off, off_chunk_bytes, off_layers, off_cand_key, off_cand_id,
      off_cand_n, off_sync, total;
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
    } else {
      return fail(IVB_EINVAL, "layer %d: unknown kind %d", i, L.kind);
    }
  }
  return IVB_OK;
}

// Builds the stream, op program and shared-memory map for a cluster of R CTAs; false if it does not fit.
static bool plan(IvbDecoder* dec, int R, size_t smem_cap, std::string& why) {
  const IvbModelDesc& md = dec->desc;
  ClusterDims& D = dec->d;
  D = ClusterDims{};
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
  D.hpc = (md.heads + R - 1) / R;
  D.taps = 1;
  D.act_eps = md.act_eps;
  D.clip = md.norm_clip;
  D.lpad = static_cast<int>(r16(md.latent_dim));
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
  const int hpc = D.hpc;
  const int dper = (d + R - 1) / R, Fper = (F + R - 1) / R, Lper = (Lt + R - 1) / R, Vper = (md.vocab + R - 1) / R;
  auto heads_of = [&](int c) { return std::max(0, std::min(H - c * hpc, hpc)); };
  auto part = [&](int n, int per, int c) { return std::max(0, std::min(n, (c + 1) * per) - std::min(n, c * per)); };
  const size_t stage = 36 * 1024;
  dec->kc = std::min(std::min(md.max_top_k, md.vocab), kMaxTopK);
  // ---- op program and per-CTA segments ------------------------------------------------------------
  struct OpPlan {
    Op op;
    std::vector<std::vector<Segment>> segs;  // [R] row segments of each CTA
    int const_kind;                           // 0 none, 1 norm, 2 mamba (norm + ssm), 3 attention
    const float* norm;
    const IvbLayerDesc* layer;
  };
  std::vector<OpPlan> plans;
  auto gemv_op = [&](int kind, int layer, const IvbTernary& m, int in_n, int rows_per, int rows_total, int gather,
                     int gather_n, int gather_per, const float* norm, float eps) {
    OpPlan pl{};
    pl.op.kind = kind;
    pl.op.layer = layer;
    pl.op.gather = gather;
    pl.op.gather_n = gather_n;
    pl.op.gather_per = gather_per;
    pl.op.in_n = in_n;
    pl.op.rows_per = rows_per;
    pl.op.rows_total = rows_total;
    pl.op.row_bytes = m.row_bytes;
    pl.op.scale_stride = ((m.in_features + 127) / 128 + 7) / 8 * 8;
    pl.op.has_bias = m.bias != nullptr;
    const int chunks = (in_n + 63) / 64;
    int lg = 0;
    while ((1 << lg) < (chunks + 2) / 3 && lg < 5) ++lg;  // at most three chunks per lane when possible
    pl.op.lpr_log = lg;
    pl.op.has_norm = norm != nullptr;
    pl.op.norm_eps = eps;
    pl.norm = norm;
    pl.const_kind = norm != nullptr ? 1 : 0;
    pl.segs.assign(R, {});
    return pl;
  };
  for (int li = 0; li < static_cast<int>(dec->layers.size()); ++li) {
    const IvbLayerDesc& L = dec->layers[li];
    const int gather0 = li == 0 ? G_NONE : G_RESID;
    if (L.kind == IVB_MAMBA) {
      OpPlan e = gemv_op(OP_ENTRY_MAMBA, li, L.entry, d, hpc * (2 * hd + 3 * S), H * (2 * hd + 3 * S), gather0, d, dper,
                         L.mixer_norm, L.mixer_norm_eps);
      e.const_kind = 2;
      e.layer = &L;
      for (int c = 0; c < R; ++c)
        for (int hl = 0; hl < heads_of(c); ++hl) {
          const int h = c * hpc + hl;
          e.segs[c].push_back({&L.entry, h * hd, hd});
          e.segs[c].push_back({&L.entry, d + h * hd, hd});
          e.segs[c].push_back({&L.entry, 2 * d + h * 3 * S, 3 * S});
        }
      plans.push_back(e);
    } else {
      OpPlan e = gemv_op(OP_ENTRY_MLA, li, L.entry, d, hpc * (hd + D.rope) + Lper, H * (hd + D.rope) + Lt, gather0, d,
                         dper, L.mixer_norm, L.mixer_norm_eps);
      e.layer = &L;
      e.op.push_per = Lper;
      for (int c = 0; c < R; ++c) {
        for (int hl = 0; hl < heads_of(c); ++hl) e.segs[c].push_back({&L.entry, (c * hpc + hl) * hd, hd});
        for (int hl = 0; hl < heads_of(c); ++hl) e.segs[c].push_back({&L.entry, d + Lt + (c * hpc + hl) * D.rope, D.rope});
        const int l0 = std::min(Lt, c * Lper), ln = part(Lt, Lper, c);
        if (ln > 0) e.segs[c].push_back({&L.entry, d + l0, ln});
      }
      plans.push_back(e);
      OpPlan a{};
      a.op.kind = OP_ATTN;
      a.op.layer = li;
      a.op.gather = G_LATENT;
      a.op.gather_n = Lt;
      a.op.gather_per = Lper;
      a.op.in_n = Lt;
      a.op.rows_per = hpc * hd;
      a.op.rows_total = d;
      a.op.lpr_log = 0;
      a.const_kind = 3;
      a.layer = &L;
      a.segs.assign(R, {});
      plans.push_back(a);
    }
    const int ygather_per = hpc * hd;
    OpPlan o = gemv_op(OP_OUT, li, L.out, d, dper, d, G_VEC, d, ygather_per, nullptr, 0.0f);
    for (int c = 0; c < R; ++c)
      if (part(d, dper, c) > 0) o.segs[c].push_back({&L.out, c * dper, part(d, dper, c)});
    plans.push_back(o);
    OpPlan g = gemv_op(OP_GATE_UP, li, L.gate_up, d, 2 * Fper, 2 * F, G_RESID, d, dper, L.ffn_norm, L.ffn_norm_eps);
    for (int c = 0; c < R; ++c)
      if (part(F, Fper, c) > 0) g.segs[c].push_back({&L.gate_up, 2 * c * Fper, 2 * part(F, Fper, c)});
    plans.push_back(g);
    OpPlan dn = gemv_op(OP_DOWN, li, L.down, F, dper, d, G_VEC, F, Fper, nullptr, 0.0f);
    for (int c = 0; c < R; ++c)
      if (part(d, dper, c) > 0) dn.segs[c].push_back({&L.down, c * dper, part(d, dper, c)});
    plans.push_back(dn);
  }
  {
    OpPlan hp = gemv_op(OP_HEAD, -1, md.head, d, Vper, md.vocab, G_RESID, d, dper, md.final_norm, md.final_norm_eps);
    for (int c = 0; c < R; ++c)
      if (part(md.vocab, Vper, c) > 0) hp.segs[c].push_back({&md.head, c * Vper, part(md.vocab, Vper, c)});
    plans.push_back(hp);
  }
  // ---- constants-chunk layouts (identical offsets for every CTA) ----------------------------------
  size_t max_const = 16;
  for (OpPlan& pl : plans) {
    Op& op = pl.op;
    size_t off = 0;
    if (pl.const_kind == 1 || pl.const_kind == 2) {
      op.c_norm = static_cast<int>(off);
      off += r16(static_cast<size_t>(d) * 4);
    }
    if (pl.const_kind == 2) {
      op.c_decay = static_cast<int>(off);
      off += r16(hpc * S * 4);
      op.c_theta = static_cast<int>(off);
      off += r16(hpc * S * 4);
      op.c_skip = static_cast<int>(off);
      off += r16(hpc * hd * 4);
      op.c_convw = static_cast<int>(off);
      off += r16(static_cast<size_t>(hpc) * hd * D.taps * 4);
      op.c_convb = static_cast<int>(off);
      off += r16(hpc * hd * 4);
    }
    if (pl.const_kind == 3) {
      op.c_wkn = static_cast<int>(off);
      off += r16(static_cast<size_t>(hpc) * D.nope * D.rb_lat);
      op.c_skn = static_cast<int>(off);
      off += r16(static_cast<size_t>(hpc) * D.nope * D.ss_lat * 2);
      op.c_bkn = static_cast<int>(off);
      off += r16(hpc * D.nope * 4);
      op.c_wv = static_cast<int>(off);
      off += r16(static_cast<size_t>(hpc) * hd * D.rb_lat);
      op.c_sv = static_cast<int>(off);
      off += r16(static_cast<size_t>(hpc) * hd * D.ss_lat * 2);
      op.c_bv = static_cast<int>(off);
      off += r16(hpc * hd * 4);
    }
    op.has_const = pl.const_kind != 0;
    max_const = std::max(max_const, off);
    pl.op.n_chunks = 0;
  }
  if (max_const > stage) {
    why = "a constants chunk does not fit a stream stage";
    return false;
  }
  // ---- chunk the rows, lay out every CTA's stream ---------------------------------------------------
  for (OpPlan& pl : plans) {
    Op& op = pl.op;
    if (op.kind == OP_ATTN) {
      op.chunk_rows = 0;
      op.n_chunks = 1;
      continue;
    }
    const size_t per_row = op.row_bytes + op.scale_stride * 2 + 4;
    int cr = static_cast<int>((stage - 64) / per_row);
    const int rpi = kThreads >> op.lpr_log;  // rows one thread-row of chunk_rows covers
    if (cr >= rpi) cr = cr / rpi * rpi;
    if (op.kind == OP_GATE_UP) cr &= ~1;
    cr = std::max(2, std::min(cr, std::max(2, op.rows_per)));
    op.chunk_rows = cr;
    op.n_chunks = op.has_const + (op.rows_per + cr - 1) / cr;
  }
  dec->ops.clear();
  dec->op_rows.assign(plans.size() * R, 0);
  int cpt = 0;
  for (size_t i = 0; i < plans.size(); ++i) {
    plans[i].op.first_chunk = cpt;
    cpt += plans[i].op.n_chunks;
    // the buffer this op waits for (filled by the previous op's pushes) and the bytes of that fill
    Op& op = plans[i].op;
    op.in_buf = XB_NONE;
    op.in_bytes = 0;
    switch (op.kind) {
      case OP_ENTRY_MAMBA:
      case OP_ENTRY_MLA:
        if (op.layer > 0) {
          op.in_buf = XB_RESID;
          op.in_bytes = d * 4;
        }
        break;
      case OP_GATE_UP:
      case OP_HEAD:
        op.in_buf = XB_RESID;
        op.in_bytes = d * 4;
        break;
      case OP_ATTN:
        op.in_buf = XB_LATENT;
        op.in_bytes = Lt * 4;
        break;
      case OP_OUT:
        op.in_buf = XB_VEC;
        op.in_bytes = H * hd * 4;
        break;
      case OP_DOWN:
        op.in_buf = XB_VEC;
        op.in_bytes = F * 4;
        break;
      default:
        break;
    }
    dec->ops.push_back(op);
  }
  dec->cpt = cpt;
  dec->head_first = plans.back().op.first_chunk;
  dec->chunk_off.assign(static_cast<size_t>(R) * cpt, 0);
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
      if (op.kind == OP_ATTN) rows_c = heads_of(c) * hd;
      dec->op_rows[i * R + c] = rows_c;
      if (op.has_const) {
        const size_t base = cursor;
        size_t bytes = 16;
        if (pl.const_kind == 1 || pl.const_kind == 2) {
          add(base + op.c_norm, pl.norm, static_cast<size_t>(d) * 4, 1, 0, 0);
          bytes = std::max(bytes, static_cast<size_t>(op.c_norm) + r16(static_cast<size_t>(d) * 4));
        }
        if (pl.const_kind == 2) {
          const IvbLayerDesc& L = *pl.layer;
          const int nh = heads_of(c), h0 = c * hpc;
          if (nh > 0) {
            add(base + op.c_decay, L.decay + h0 * S, nh * S * 4, 1, 0, 0);
            add(base + op.c_theta, L.theta + h0 * S, nh * S * 4, 1, 0, 0);
            add(base + op.c_skip, L.skip + h0 * hd, nh * hd * 4, 1, 0, 0);
            add(base + op.c_convw, L.conv_weight + static_cast<size_t>(h0) * hd * D.taps, static_cast<size_t>(nh) * hd * D.taps * 4, 1, 0, 0);
            add(base + op.c_convb, L.conv_bias + h0 * hd, nh * hd * 4, 1, 0, 0);
          }
          bytes = std::max(bytes, static_cast<size_t>(op.c_convb) + r16(hpc * hd * 4));
        }
        if (pl.const_kind == 3) {
          const IvbLayerDesc& L = *pl.layer;
          const int nh = heads_of(c), h0 = c * hpc;
          const IvbTernary& kn = L.k_nope_up;
          const IvbTernary& vu = L.v_up;
          const size_t sgroups = static_cast<size_t>((Lt + 127) / 128) * 2;
          if (nh > 0) {
            add(base + op.c_wkn, kn.packed + static_cast<size_t>(h0) * D.nope * kn.row_bytes, D.rb_lat, nh * D.nope, kn.row_bytes, D.rb_lat);
            add(base + op.c_skn, kn.scales + static_cast<size_t>(h0) * D.nope * kn.scale_stride, sgroups, nh * D.nope,
                static_cast<size_t>(kn.scale_stride) * 2, static_cast<size_t>(D.ss_lat) * 2);
            add(base + op.c_bkn, kn.bias ? static_cast<const void*>(kn.bias + h0 * D.nope) : nullptr, nh * D.nope * 4, 1, 0, 0);
            add(base + op.c_wv, vu.packed + static_cast<size_t>(h0) * hd * vu.row_bytes, D.rb_lat, nh * hd, vu.row_bytes, D.rb_lat);
            add(base + op.c_sv, vu.scales + static_cast<size_t>(h0) * hd * vu.scale_stride, sgroups, nh * hd,
                static_cast<size_t>(vu.scale_stride) * 2, static_cast<size_t>(D.ss_lat) * 2);
            add(base + op.c_bv, vu.bias ? static_cast<const void*>(vu.bias + h0 * hd) : nullptr, nh * hd * 4, 1, 0, 0);
          }
          bytes = std::max(bytes, static_cast<size_t>(op.c_bv) + r16(hpc * hd * 4));
        }
        dec->chunk_off[static_cast<size_t>(c) * cpt + ci] = base;
        dec->chunk_bytes[static_cast<size_t>(c) * cpt + ci] = static_cast<unsigned>(r16(bytes));
        cursor = r16(base + bytes);
        ++ci;
      }
      if (op.kind == OP_ATTN) continue;
      // row chunks: [k x row_bytes][k x scale_stride fp16, 16B pad][k x fp32 bias, 16B pad]
      const int n_row_chunks = op.n_chunks - op.has_const;
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
            add(base + dr * op.row_bytes, m.packed + static_cast<size_t>(src_row) * m.row_bytes, op.row_bytes, n, m.row_bytes,
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
  dec->stream_bytes = r16(cursor) + 256;
  // ---- shared memory map ----------------------------------------------------------------------------
  ClusterSmem& M = dec->sm;
  size_t o = 0;
  M.ring = 0;
  M.stage_bytes = static_cast<int>(stage);
  o += kStages * stage;
  const int max_in = std::max(d, F);
  const int pad_in = (max_in + 63) / 64 * 64;
  M.xv = static_cast<int>(o);
  o += r16(static_cast<size_t>(pad_in) * 4);
  M.act = static_cast<int>(o);
  o += r16(pad_in);
  M.xsum = static_cast<int>(o);
  o += r16(pad_in / 64 * 4);
  M.resid = static_cast<int>(o);
  o += r16(static_cast<size_t>(d) * 4);
  int pub_n = std::max(std::max(hpc * hd, Lper), std::max(dper, Fper));
  M.pub_n = pub_n;
  M.pub = static_cast<int>(o);
  o += r16(static_cast<size_t>(pub_n) * 4);  // staging of the op's output slice
  int loc_n = 0;
  for (const Op& op : dec->ops) loc_n = std::max(loc_n, op.kind == OP_ATTN ? 0 : op.rows_per);
  M.loc = static_cast<int>(o);
  o += r16(static_cast<size_t>(loc_n) * 4);
  M.red = static_cast<int>(o);
  o += r16(64 * 4);
  M.xl = static_cast<int>(o);
  o += r16(static_cast<size_t>((Lt + 63) / 64 * 64) * 4);
  M.ctab = static_cast<int>(o);
  o += r16(static_cast<size_t>(dec->cpt) * 8) + r16(static_cast<size_t>(dec->cpt) * 4);
  M.rope_row = static_cast<int>(o);
  o += r16(static_cast<size_t>(std::max(md.rope_dim, 1)) * 4);
  M.seen = static_cast<int>(o);
  o += r16(static_cast<size_t>(Vper));
  M.u = static_cast<int>(o);
  const int kc = dec->kc;
  // recurrent op: constants, coefficients, values, partial readouts, prefetched state
  size_t u_need = r16((static_cast<size_t>(ssm_const_floats(hpc, S, hd, D.taps)) + 5 * hpc * S + hpc * hd + std::max(kThreads, hpc * hd) +
                       3 * static_cast<size_t>(hpc) * S * hd + static_cast<size_t>(hpc) * hd * (D.taps - 1)) * 4);
  // head + sampler: the head's top-k scratch (or the merge scratch) first, then the merge arrays that
  // the other CTAs push their candidates into
  const size_t head_scratch = static_cast<size_t>(Vper) * 4 + 4 * static_cast<size_t>(kc) * 4 + kWarps * 256 * 4 + 16 * 4;
  const size_t merge_scratch = 5 * static_cast<size_t>(kc) * 4 + kWarps * 256 * 4 + 16 * 4;
  M.cand = static_cast<int>(r16(std::max(head_scratch, merge_scratch)));
  u_need = std::max(u_need, static_cast<size_t>(M.cand) + 2 * r16(static_cast<size_t>(R) * kc * 4));
  const size_t attn_fixed = r16(static_cast<size_t>((Lt + 63) / 64 * 64) * 4) + r16((Lt + 63) / 64 * 64) +
                            static_cast<size_t>(Lt + 2 * D.rope + D.nope) * 4 + kWarps * Lt * 4 + 64;
  const size_t per_pos = static_cast<size_t>(D.lpad) + 4 + static_cast<size_t>(D.rpad) * 2;
  bool any_mla = false;
  for (const IvbLayerDesc& L : dec->layers) any_mla |= L.kind == IVB_MLA;
  int tile = 0;
  if (any_mla) {
    const size_t room = smem_cap > o + attn_fixed ? smem_cap - o - attn_fixed : 0;
    tile = static_cast<int>(room / (2 * per_pos + 8)) / 16 * 16;
    tile = std::min(tile, (md.max_len + 15) / 16 * 16);
    if (tile < 16) {
      why = "no room for an attention tile in shared memory";
      return false;
    }
    tile = std::min(tile, 512);
    u_need = std::max(u_need, attn_fixed + static_cast<size_t>(tile) * 4 + 64 + 2 * (r16(static_cast<size_t>(tile) * D.lpad) +
                                                                                  r16(tile * 4) + r16(static_cast<size_t>(tile) * D.rpad * 2)));
  }
  D.tile = std::max(tile, 16);
  o += r16(u_need);
  M.total = static_cast<int>(o);
  if (o > smem_cap) {
    why = "the cluster decoder needs more shared memory than a CTA has";
    return false;
  }
  dec->smem = o;
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
  int dev = 0, optin = 0;
  IVB_CUDA(cudaGetDevice(&dev));
  IVB_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  const size_t cap = static_cast<size_t>(optin) - 4096;  // static shared memory of the kernel
  IVB_CUDA(cudaFuncSetAttribute(cluster_decode_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  std::string why = "no cluster size fits";
  bool planned = false;
  for (int R : {16, 8, 4, 2, 1}) {
    if (ctas > 0 && R > ctas) continue;
    if (!plan(dec, R, cap, why)) continue;
    IVB_CUDA(cudaFuncSetAttribute(cluster_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dec->smem)));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(R);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = dec->smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = R;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, reinterpret_cast<const void*>(cluster_decode_kernel), &cfg) != cudaSuccess ||
        clusters < 1) {
      cudaGetLastError();
      why = "the device cannot schedule the cluster";
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
  const int R = dec->R;
  size_t off = 0;
  dec->off_stream = off;
  off = align_up(off + dec->stream_bytes, 256);
  dec->off_ops = off;
  off = align_up(off + dec->ops.size() * sizeof(OpRec), 256);
  dec->off_op_rows = off;
  off = align_up(off + dec->op_rows.size() * 4, 256);
  dec->off_chunk_off = off;
  off = align_up(off + dec->chunk_off.size() * 8, 256);
  dec->off_chunk_bytes = off;
  off = align_up(off + dec->chunk_bytes.size() * 4, 256);
  dec->off_layers = off;
  off = align_up(off + dec->layers.size() * sizeof(IvbLayerDesc), 256);
  dec->off_cand_key = off;
  off = align_up(off + static_cast<size_t>(R) * dec->kc * 4, 256);
  dec->off_cand_id = off;
  off = align_up(off + static_cast<size_t>(R) * dec->kc * 4, 256);
  dec->off_cand_n = off;
  off = align_up(off + R * 4, 256);
  dec->off_sync = off;
  off = align_up(off + 256, 256);
  dec->total = off;
  *out = dec;
  return IVB_OK;
}

void ivb_decoder_destroy(IvbDecoder* dec) { delete dec; }

uint64_t ivb_decoder_workspace_bytes(const IvbDecoder* dec) { return dec ? dec->total : 0; }

int32_t ivb_decoder_num_phases(const IvbDecoder* dec) { return dec ? static_cast<int32_t>(dec->ops.size()) : 0; }

int32_t ivb_decoder_ctas(const IvbDecoder* dec) { return dec ? dec->R : 0; }

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
  IVB_CUDA(cudaMemcpyAsync(ws + dec->off_op_rows, dec->op_rows.data(), dec->op_rows.size() * 4, cudaMemcpyHostToDevice, s));
  IVB_CUDA(cudaMemcpyAsync(ws + dec->off_chunk_off, dec->chunk_off.data(), dec->chunk_off.size() * 8, cudaMemcpyHostToDevice, s));
  IVB_CUDA(cudaMemcpyAsync(ws + dec->off_chunk_bytes, dec->chunk_bytes.data(), dec->chunk_bytes.size() * 4, cudaMemcpyHostToDevice, s));
  IVB_CUDA(cudaMemcpyAsync(ws + dec->off_layers, dec->layers.data(), dec->layers.size() * sizeof(IvbLayerDesc),
                           cudaMemcpyHostToDevice, s));
  IVB_CUDA(cudaMemsetAsync(ws + dec->off_cand_n, 0, dec->R * 4, s));
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
  ClusterParams p{};
  p.ops = reinterpret_cast<const OpRec*>(ws + dec->off_ops);
  p.op_rows = reinterpret_cast<const int32_t*>(ws + dec->off_op_rows);
  p.n_ops = static_cast<int32_t>(dec->ops.size());
  p.kc = dec->kc;
  p.head_first = dec->head_first;
  p.chunks_per_token = dec->cpt;
  p.steps = steps;
  p.chunk_off = reinterpret_cast<const unsigned long long*>(ws + dec->off_chunk_off);
  p.chunk_bytes = reinterpret_cast<const unsigned*>(ws + dec->off_chunk_bytes);
  p.stream = ws + dec->off_stream;
  p.d = dec->d;
  p.sm = dec->sm;
  p.layers = reinterpret_cast<const IvbLayerDesc*>(ws + dec->off_layers);
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
  p.cand_key = reinterpret_cast<unsigned*>(ws + dec->off_cand_key);
  p.cand_id = reinterpret_cast<int*>(ws + dec->off_cand_id);
  p.cand_n = reinterpret_cast<int*>(ws + dec->off_cand_n);
  p.error = error;
  p.feed = feed;
  p.timeout_ns = timeout_ns == 0 ? 1000000000ull : timeout_ns;
  p.trace = dec->trace;
  p.trace_step = dec->trace_step;
  p.flags = flags;
  IVB_CUDA(cudaMemsetAsync(error, 0, 4, s));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(dec->R);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = dec->smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = dec->R;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  IVB_CUDA(cudaLaunchKernelEx(&cfg, cluster_decode_kernel, p));
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
