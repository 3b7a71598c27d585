// Prefill ternary GEMM of libivonar_b200.so on the 5th-generation tensor cores (tcgen05, kind::i8).
//
// out[t][r] = epilogue(act_scale[t] * sum_g s[r][g] * (sum_{k in g} (code[r][k] - 1) * q8[t][k]) + bias[r])
// for T token rows at once: the per-group integer dot is exact in the int32 accumulator, then scaled by
// the fp16 group scale in fp32. Reference: kernels/ternary.cu:688-765 gemm_tile_body (per-token int8
// tiles, dp4a), which subtracts the activation group sum instead of offsetting the codes.
//
// Persistent: one CTA per SM walks units of 128 weight rows x 128 tokens (x one split of K), and every
// role keeps a running group count over the CTA's whole sequence, so the next unit's copies, expansion
// and MMAs overlap the current unit's epilogue. The weights are the MMA's A operand and live in tensor
// memory: they never pass through shared memory as expanded bytes. Warp-specialised roles per
// 128-input group G:
//   * a copy warp (one thread) issues every copy up to eight groups ahead: the unit's packed weights of
//     the group (128 rows x 32 bytes) with one TMA tensor load into a packed ring, and the group's 16 KB
//     activation tile (core matrices, laid out by ivb_quantize_rows) with one bulk copy into an
//     8-stage ring;
//   * two producer teams of 4 warps (one TMEM lane quarter each), team t expanding the groups
//     G = t (mod 2): every thread turns its row's 128 two-bit codes into signed bytes (code - 1) in
//     registers and stores them into A slot G % 4 in TMEM (tcgen05.st, 32 columns);
//   * one MMA thread: four 128x128x32 int8 MMAs (A from TMEM, B = activations from shared memory) into
//     TMEM accumulator G % 3, committed to the stage's, the A slot's and the accumulator's barriers;
//   * epilogue warps (16; warp w reads TMEM lane quarter w % 4 = weight rows, columns 32 (w / 4).. =
//     tokens): drain the accumulator (tcgen05.ld), recover the exact int32 group dots from the biased
//     accumulator, scale them by the row's group scale and accumulate in fp32 registers (paired
//     multiply-adds); at the end of a unit, store the outputs straight from registers.
// TMEM: 3 accumulators x 128 columns + 4 A slots x 32 columns = all 512 columns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "ivb_common.h"
#include "ivb_decode.cuh"
#include "ivb_tc.cuh"
#include "ivb_tiles.cuh"

namespace ivb {

constexpr int kGemmRows = 128;       // weight rows per tile (MMA M, TMEM lanes)
constexpr int kGemmTok = 128;        // tokens per tile (MMA N, accumulator columns)
constexpr int kGemmStages = 8;       // activation stages in shared memory (groups copied ahead)
constexpr int kGemmASlots = 4;       // TMEM A slots of 32 columns (expanded groups in flight)
constexpr int kGemmBufs = 3;         // TMEM accumulators of 128 columns
constexpr int kGemmACol = kGemmBufs * kGemmTok;  // first TMEM column of the A slots
constexpr int kGemmEpiWarps = 16;    // warps 0-15: epilogue
constexpr int kGemmEpiCols = 32;     // accumulator columns (tokens) per epilogue thread
constexpr int kGemmMmaWarp = 16;     // warp 16: TMEM allocation and the MMA thread
constexpr int kGemmTeams = 2;        // producer teams: team t expands the groups G = t (mod 2)
constexpr int kGemmProdWarps = 4 * kGemmTeams;  // warps 17-24: producers (lane quarter = warp % 4)
constexpr int kGemmProducers = 128;  // threads of one team (one per weight row / TMEM lane)
constexpr int kGemmLoadWarp = kGemmMmaWarp + 1 + kGemmProdWarps;  // warp 25: lane 0 issues every copy
constexpr int kGemmThreads = 32 * (kGemmLoadWarp + 1);
constexpr int kPackSlots = 8;                    // packed weight blocks in flight
constexpr int kPackSlot = kGemmRows * 32;        // packed bytes of one group for the tile's 128 rows
constexpr uint32_t kAccBias = 0x4B400000u;       // accumulator start value: the float 12582912 as an integer

// kind::i8 instruction descriptor: D s32, A s8 (weight codes - 1, TMEM), B s8 (activations, shared
// memory), both K-major, M 128, N 128.
constexpr uint32_t kGemmIdesc = (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kGemmTok >> 3) << 17) |
                                (static_cast<uint32_t>(kGemmRows >> 4) << 24);

// TMA tensor load of a 2-D box (x: byte column, y: row) of the packed weights into shared memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}
// Persistent: grid = min(units, SMs); CTA b takes the units b, b + gridDim.x, ... A unit is one
// (row tile x, token tile y, split z) with x fastest. Every role walks the same sequence of (unit, group)
// pairs, and its running group count G picks the ring entries and their phases, so the copies and
// expansions of the next unit overlap the current unit's last MMAs and its epilogue.
// q8: the tiled activation layout (q8_chunk_offset), act_scale [T]; wmap: 2-D tensor map over the packed
// weights (row_bytes x rows bytes, box 32 x 128).
struct GemmUnit {
  int r0, t0, z, g_lo, groups;
};

__device__ __forceinline__ GemmUnit gemm_unit(int u, int row_tiles, int tok_tiles, int g_per, int groups_all) {
  GemmUnit w;
  const int per_z = row_tiles * tok_tiles;
  w.z = u / per_z;
  const int rest = u - w.z * per_z;
  const int y = rest / row_tiles;
  w.r0 = (rest - y * row_tiles) * kGemmRows;
  w.t0 = y * kGemmTok;
  w.g_lo = w.z * g_per;
  w.groups = max(0, min(groups_all, w.g_lo + g_per) - w.g_lo);
  return w;
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    ternary_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const IvbTernary m, const int8_t* __restrict__ q8,
                        int ldq, const float* __restrict__ act_scale, int T, int epilogue, float* out, int ldo,
                        int g_per, int row_tiles, int tok_tiles, int units, float* partial,
                        unsigned long long timeout_ns, unsigned* error) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      smem_raw + ((1024u - (static_cast<unsigned>(__cvta_generic_to_shared(smem_raw)) & 1023u)) & 1023u);
  // act_full/act_empty: activation stages (loader -> MMA); a_full/a_empty: TMEM A slots (producers ->
  // MMA); tfull/tempty: accumulators (MMA -> epilogue); pk_bar/pk_empty: packed weights (loader ->
  // producers)
  __shared__ __align__(8) unsigned long long act_full[kGemmStages], act_empty[kGemmStages];
  __shared__ __align__(8) unsigned long long a_full[kGemmASlots], a_empty[kGemmASlots];
  __shared__ __align__(8) unsigned long long tfull_bar[kGemmBufs], tempty_bar[kGemmBufs];
  __shared__ __align__(8) unsigned long long pk_bar[kPackSlots], pk_empty[kPackSlots];
  __shared__ unsigned tmem_base;
  __shared__ int failed;
  __shared__ int stage_group[kGemmStages], slot_group[kPackSlots];  // last group copied into each (error drain)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int groups_all = (m.in_features + 127) >> 7;
  unsigned char* pack = smem + kGemmStages * kGemmTile;  // packed ring
  const bool loader = tid == 32 * kGemmLoadWarp;
  unsigned pre = 0;  // loader: packed-weight groups copied before the wait for the previous kernel
  if (warp == kGemmMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (loader) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&wmap) : "memory");
    for (int i = 0; i < kGemmStages; ++i) {
      mbar_init(act_full + i, 1);
      mbar_init(act_empty + i, 1);
      stage_group[i] = -1;
    }
    for (int i = 0; i < kGemmASlots; ++i) {
      mbar_init(a_full + i, kGemmProducers);
      mbar_init(a_empty + i, 1);
    }
    for (int i = 0; i < kGemmBufs; ++i) {
      mbar_init(tfull_bar + i, 1);
      mbar_init(tempty_bar + i, kGemmEpiWarps);
    }
    for (int i = 0; i < kPackSlots; ++i) {
      mbar_init(pk_bar + i, 1);
      mbar_init(pk_empty + i, kGemmProducers);
      slot_group[i] = -1;
    }
    failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    {
      // the packed weights do not depend on the previous kernel: the first unit's first four groups
      // are copied before the wait for it below
      const GemmUnit w = gemm_unit(blockIdx.x, row_tiles, tok_tiles, g_per, groups_all);
      for (int g = 0; g < w.groups && pre < 4; ++g, ++pre) {
        slot_group[pre] = static_cast<int>(pre);
        mbar_expect_tx(pk_bar + pre, kPackSlot);
        tma_load_2d(pack + pre * kPackSlot, &wmap, (w.g_lo + g) << 5, w.r0, pk_bar + pre);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // launched as a programmatic dependent: the set-up above may overlap the previous kernel; its outputs
  // (activations, scales, a residual to add to) are read only after this wait
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const unsigned tmem = tmem_base;
  const int quarter = warp & 3;               // TMEM lane quarter this warp may access
  const int row = 32 * quarter + lane;        // epilogue and producer warps: the weight row (TMEM lane)
  const unsigned lane_base = tmem + (static_cast<unsigned>(32 * quarter) << 16);
  const int col0 = (warp >> 2) * kGemmEpiCols;  // epilogue warps: first token column
  volatile int* fail_flag = &failed;
  bool late = false;
  unsigned G = 0;  // groups of this CTA's sequence handled so far (by this role)

  if (warp == kGemmLoadWarp) {
    // ---- loader: every copy, up to kGemmStages groups of activations and kPackSlots of packed weights
    // ahead of the MMA ----
    if (lane == 0) {
      for (int u = blockIdx.x; u < units && !late; u += gridDim.x) {
        const GemmUnit w = gemm_unit(u, row_tiles, tok_tiles, g_per, groups_all);
        const int8_t* a_src = q8 + static_cast<size_t>(w.t0 >> 7) * (ldq >> 7) * kGemmTile;
        for (int g = 0; g < w.groups; ++g, ++G) {
          const int st = G % kGemmStages, slot = G % kPackSlots;
          if (*fail_flag || (G >= kGemmStages && !mbar_wait_bounded(act_empty + st, ((G / kGemmStages) - 1) & 1, timeout_ns))) {
            late = true;
            break;
          }
          stage_group[st] = static_cast<int>(G);
          mbar_expect_tx(act_full + st, kGemmTile);
          bulk_copy(smem + st * kGemmTile, a_src + static_cast<size_t>(w.g_lo + g) * kGemmTile, kGemmTile, act_full + st);
          if (G < pre) continue;  // its packed weights were copied before the wait
          if (G >= kPackSlots && !mbar_wait_bounded(pk_empty + slot, ((G / kPackSlots) - 1) & 1, timeout_ns)) {
            late = true;
            break;
          }
          slot_group[slot] = static_cast<int>(G);
          mbar_expect_tx(pk_bar + slot, kPackSlot);
          tma_load_2d(pack + slot * kPackSlot, &wmap, (w.g_lo + g) << 5, w.r0, pk_bar + slot);
        }
      }
      if (late) atomicExch(&failed, 1);
    }
    __syncwarp();
  } else if (warp > kGemmMmaWarp) {
    // ---- producers: team `team` expands the groups G = team (mod 2) into TMEM A slot G % 4 ----
    const int team = (warp - kGemmMmaWarp - 1) >> 2;
    for (int u = blockIdx.x; u < units && !late; u += gridDim.x) {
      const GemmUnit w = gemm_unit(u, row_tiles, tok_tiles, g_per, groups_all);
      for (int g = 0; g < w.groups; ++g, ++G) {
        if ((G & 1u) != static_cast<unsigned>(team)) continue;
        const int slot = G % kPackSlots, as = G % kGemmASlots;
        if (*fail_flag || !mbar_wait_bounded(pk_bar + slot, (G / kPackSlots) & 1, timeout_ns) ||
            (G >= kGemmASlots && !mbar_wait_bounded(a_empty + as, ((G / kGemmASlots) - 1) & 1, timeout_ns))) {
          late = true;
          break;
        }
        // row's 16 packed words -> 32 TMEM columns: column 4c + f holds the codes (w_c >> 2f) & 0x03030303
        // (inputs 16c + 4b + f, b = 0..3), each byte turned into the signed code - 1
        const uint4* pk = reinterpret_cast<const uint4*>(pack + slot * kPackSlot + row * 32);
        const uint4 p0 = pk[0], p1 = pk[1];
        const uint32_t words[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        uint32_t v[32];
#pragma unroll
        for (int c = 0; c < 8; ++c)
#pragma unroll
          for (int f = 0; f < 4; ++f) v[4 * c + f] = (((words[c] >> (2 * f)) & 0x03030303u) + 0x7F7F7F7Fu) ^ 0x80808080u;
        mbar_arrive(pk_empty + slot);
        tmem_st32(lane_base + kGemmACol + as * 32, v);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(a_full + as);
      }
    }
    if (late) atomicExch(&failed, 1);
  } else if (warp == kGemmMmaWarp) {
    // ---- MMA issuer: group G = four 128x128x32 int8 MMAs into accumulator G % 3 ----
    int last = -1;  // accumulator of the last group issued (the exit waits for its MMAs)
    unsigned last_g = 0;
    if (lane == 0) {
      for (int u = blockIdx.x; u < units && !late; u += gridDim.x) {
        const GemmUnit w = gemm_unit(u, row_tiles, tok_tiles, g_per, groups_all);
        for (int g = 0; g < w.groups; ++g, ++G) {
          const int st = G % kGemmStages, as = G % kGemmASlots, b = G % kGemmBufs;
          // tempty completion k of accumulator b: armed for group b + 3k (k = 0: the initial arming)
          if (*fail_flag || !mbar_wait_bounded(act_full + st, (G / kGemmStages) & 1, timeout_ns) ||
              !mbar_wait_bounded(a_full + as, (G / kGemmASlots) & 1, timeout_ns) ||
              !mbar_wait_bounded(tempty_bar + b, (G / kGemmBufs) & 1, timeout_ns)) {
            late = true;
            break;
          }
          tc_fence_after();
          const unsigned bsm = smem_addr(smem + st * kGemmTile);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_i8_ta(tmem + b * kGemmTok, tmem + kGemmACol + as * 32 + kk * 8, smem_desc(bsm + kk * 256), kGemmIdesc, true);
          umma_commit(act_empty + st);
          umma_commit(a_empty + as);
          umma_commit(tfull_bar + b);
          last = b;
          last_g = G;
        }
      }
      if (late) atomicExch(&failed, 1);
      // no MMA may still be writing tensor memory when it is released
      if (last >= 0) mbar_wait_bounded(tfull_bar + last, (last_g / kGemmBufs) & 1, timeout_ns);
    }
    __syncwarp();
  } else {
    // ---- epilogue: drain, scale, accumulate; then write the unit's outputs straight from registers ----
    // Exact int32 -> float without a conversion: every accumulator starts a group holding the integer
    // 0x4B400000 and the MMAs add the group's dot to it, so its bits are the float 12582912 + dot
    // (|dot| <= 128 * 127 < 2^22 keeps it in [2^23, 2^24), where float steps are 1); one paired
    // subtract leaves dot. The drain puts the start value back for the accumulator's next group.
    for (int b = 0; b < kGemmBufs; ++b) tmem_fill32(lane_base + b * kGemmTok + col0, kAccBias);
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0)
      for (int b = 0; b < kGemmBufs; ++b) mbar_arrive(tempty_bar + b);
    const float2 m2 = make_float2(-12582912.0f, -12582912.0f);
    for (int u = blockIdx.x; u < units && !late; u += gridDim.x) {
      const GemmUnit w = gemm_unit(u, row_tiles, tok_tiles, g_per, groups_all);
      const int r = w.r0 + row;
      const uint16_t* srow = r < m.rows ? m.scales + static_cast<size_t>(r) * m.scale_stride + w.g_lo : nullptr;
      float2 acc[kGemmEpiCols / 2];
#pragma unroll
      for (int n = 0; n < kGemmEpiCols / 2; ++n) acc[n] = make_float2(0.0f, 0.0f);
      // the row's group scales, loaded two groups ahead of their use
      float s_cur = srow != nullptr && w.groups > 0 ? h2f(__ldg(srow)) : 0.0f;
      float s_nxt = srow != nullptr && w.groups > 1 ? h2f(__ldg(srow + 1)) : 0.0f;
      // the unit's per-token and per-row epilogue inputs, loaded before the drain so their latency hides
      // behind it: lane l holds act_scale of token t0 + col0 + l
      const int tb = w.t0 + col0;
      const int nt = min(kGemmEpiCols, T - tb);  // tokens of this warp's columns that exist
      const float asc = partial == nullptr && lane < nt ? __ldg(act_scale + tb + lane) : 0.0f;
      const float bias_r = partial == nullptr && m.bias != nullptr && r < m.rows ? __ldg(m.bias + r) : 0.0f;
      for (int g = 0; g < w.groups; ++g, ++G) {
        const int b = G % kGemmBufs;
        const float s_far = srow != nullptr && g + 2 < w.groups ? h2f(__ldg(srow + g + 2)) : 0.0f;
        late = !mbar_wait_bounded(tfull_bar + b, (G / kGemmBufs) & 1, timeout_ns);
        if (__any_sync(kFull, late)) {
          late = true;
          break;
        }
        tc_fence_after();
        const float2 s2 = make_float2(s_cur, s_cur);
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          uint32_t d[8];
          tmem_ld8(lane_base + b * kGemmTok + col0 + 8 * h, d);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 x = __fadd2_rn(make_float2(__uint_as_float(d[2 * q]), __uint_as_float(d[2 * q + 1])), m2);
            acc[4 * h + q] = __ffma2_rn(x, s2, acc[4 * h + q]);
          }
          tmem_fill8(lane_base + b * kGemmTok + col0 + 8 * h, kAccBias);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty_bar + b);
        s_cur = s_nxt;
        s_nxt = s_far;
      }
      if (late) break;
      // token t = t0 + col0 + j of this warp: its 32 lanes hold 32 consecutive weight rows, so every
      // store below is one contiguous 128-byte (64-byte for silu pairs) run per warp. All 32 columns are
      // evaluated without a branch, so that the unrolled iterations overlap; tokens past T are not stored.
      if (partial == nullptr && epilogue == IVB_EPI_SILU_PAIR) {
        // tokens j (even) and j + 1 at once: rows 2i (gate) and 2i + 1 (up) of token j go to lane i,
        // those of token j + 1 to lane 16 + i, so each lane evaluates one silu per two tokens
        const int src = 2 * (lane & 15), rg = w.r0 + 32 * quarter + src;
        const bool second = lane >= 16;
#pragma unroll
        for (int j = 0; j < kGemmEpiCols; j += 2) {
          const float v0 = acc[j >> 1].x * __shfl_sync(kFull, asc, j) + bias_r;
          const float v1 = acc[j >> 1].y * __shfl_sync(kFull, asc, j + 1) + bias_r;
          const float g0 = __shfl_sync(kFull, v0, src), u0 = __shfl_sync(kFull, v0, src + 1);
          const float g1 = __shfl_sync(kFull, v1, src), u1 = __shfl_sync(kFull, v1, src + 1);
          const int jj = j + (second ? 1 : 0);
          if (jj < nt && rg + 1 < m.rows)
            out[static_cast<size_t>(tb + jj) * ldo + (rg >> 1)] = silu_f(second ? g1 : g0) * (second ? u1 : u0);
        }
      } else {
        // four tokens at a time so that a residual's loads are issued together
#pragma unroll
        for (int jb = 0; jb < kGemmEpiCols; jb += 4) {
          float old[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            old[e] = epilogue == IVB_EPI_RESIDUAL && partial == nullptr && jb + e < nt && r < m.rows
                         ? out[static_cast<size_t>(tb + jb + e) * ldo + r]
                         : 0.0f;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = jb + e;
            const float a = (j & 1) ? acc[j >> 1].y : acc[j >> 1].x;
            const float sc = __shfl_sync(kFull, asc, j);
            const size_t t = static_cast<size_t>(tb + j);
            if (j >= nt || r >= m.rows) continue;
            if (partial != nullptr) {  // split-K: this split's raw sums; scale, bias and epilogue in the reduction
              partial[(static_cast<size_t>(w.z) * T + t) * m.rows + r] = a;
            } else {
              const float v = a * sc + bias_r;
              out[t * ldo + r] = epilogue == IVB_EPI_RESIDUAL ? old[e] + v : v;
            }
          }
        }
      }
    }
    if (late && lane == 0) atomicExch(&failed, 1);
  }
  __syncthreads();
  if (failed != 0) {
    if (tid == 0) atomicCAS(error, 0u, static_cast<unsigned>(IVB_ETIMEOUT));
    // no bulk or tensor copy may still be writing this CTA's shared memory when it exits
    if (loader) {
      for (int i = 0; i < kGemmStages; ++i)
        if (stage_group[i] >= 0) mbar_wait_bounded(act_full + i, (stage_group[i] / kGemmStages) & 1, timeout_ns);
      for (int i = 0; i < kPackSlots; ++i)
        if (slot_group[i] >= 0) mbar_wait_bounded(pk_bar + i, (slot_group[i] / kPackSlots) & 1, timeout_ns);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kGemmMmaWarp) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}

// Split-K reduction: out = epilogue(act_scale[t] * sum_z partial[z][t][r] + bias[r]), splits summed in order.
__global__ void gemm_splitk_reduce_kernel(const float* partial, int splits, int T, int rows, const float* act_scale,
                                          const float* bias, int epilogue, float* out, int ldo) {
  pdl_enter();
  const int per_row = epilogue == IVB_EPI_SILU_PAIR ? rows / 2 : rows;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * per_row) return;
  const int t = i / per_row, j = i - t * per_row;
  const float sc = __ldg(act_scale + t);
  auto value = [&](int r) {
    float v = 0.0f;
    for (int z = 0; z < splits; ++z) v += partial[(static_cast<size_t>(z) * T + t) * rows + r];
    v *= sc;
    if (bias != nullptr) v += __ldg(bias + r);
    return v;
  };
  float* orow = out + static_cast<size_t>(t) * ldo;
  if (epilogue == IVB_EPI_SILU_PAIR) {
    orow[j] = silu_f(value(2 * j)) * value(2 * j + 1);
  } else {
    const float v = value(j);
    orow[j] = epilogue == IVB_EPI_RESIDUAL ? orow[j] + v : v;
  }
}

// Partial sums of split-K calls of the public ivb_ternary_gemm (token counts too small to fill the GPU
// with row tiles): a file-scope device scratch, so the entry point allocates nothing; calls on one device
// use it one at a time. The prefill and the batched decode bring their own (ternary_gemm_into).
static __device__ __align__(256) float g_gemm_partial[kGemmPartialFloats];

// One CTA per token row: the canonical quantiser (RMSNorm optional), codes written as 16-byte chunks of
// the tiled GEMM activation layout (q8_chunk_offset, gemm_slot order inside a chunk), per-128-group sums
// of the codes.
__global__ void __launch_bounds__(kThreads) quantize_rows_kernel(const float* x, int n, const float* norm_w, float norm_eps,
                                                                 float clip, float act_eps, int8_t* q8, int ldq,
                                                                 float* scale, int32_t* gsum) {
  pdl_enter();  // the next kernel (a GEMM) may start its set-up now; it waits for this grid's completion
  extern __shared__ __align__(16) unsigned char smem[];
  const int pad = ((n + 63) >> 6) << 6;
  float* xv = reinterpret_cast<float*>(smem);
  int8_t* codes = reinterpret_cast<int8_t*>(xv + pad);
  float* red = reinterpret_cast<float*>(codes + pad);
  const int row = blockIdx.x;
  load_vector(x + static_cast<size_t>(row) * n, n, xv);
  __syncthreads();
  const float s = quantize_block(xv, n, norm_w, norm_eps, clip, act_eps, codes, false, nullptr, red);
  const int groups = (n + 127) >> 7;
  for (int k = threadIdx.x; k < (ldq >> 4); k += kThreads) {
    // word f, byte b of chunk k holds input 16k + 4b + f
    uint32_t o[4];
#pragma unroll
    for (int f = 0; f < 4; ++f) {
      uint32_t w = 0u;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int i = (k << 4) + 4 * b + f;
        w |= (i < n ? static_cast<uint32_t>(static_cast<uint8_t>(codes[i])) : 0u) << (8 * b);
      }
      o[f] = w;
    }
    *reinterpret_cast<uint4*>(q8 + q8_chunk_offset(row, k, ldq)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  // group sums: one warp per group, exact integers
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int g = warp; gsum != nullptr && g < groups; g += kWarps) {
    int sum = 0;
    for (int i = (g << 7) + lane; i < min(n, (g + 1) << 7); i += 32) sum += codes[i];
    sum = __reduce_add_sync(kFull, sum);
    if (lane == 0) gsum[static_cast<size_t>(row) * groups + g] = sum;
  }
  if (threadIdx.x == 0) scale[row] = s;
}

// Per-row max |x|.
__global__ void __launch_bounds__(kThreads) rows_amax_kernel(const float* x, int n, float* amax) {
  pdl_enter();
  __shared__ float red[64];
  const float* row = x + static_cast<size_t>(blockIdx.x) * n;
  float am = 0.0f;
  for (int i = threadIdx.x; i < n; i += kThreads) am = fmaxf(am, fabsf(row[i]));
  const float m = block_max_nonneg(am, red);
  if (threadIdx.x == 0) amax[blockIdx.x] = m;
}

// The quantiser without RMSNorm for a given amax per row (the whole row's, for a shard), codes in the
// tiled GEMM layout: scale = max(amax / 127, act_eps), code = rint(x / scale) (the decode quantiser's
// fast reciprocal path with its exact fallback near half-integers).
__global__ void __launch_bounds__(kThreads) quantize_rows_amax_kernel(const float* x, int n, const float* amax_in,
                                                                      float act_eps, int8_t* q8, int ldq, float* scale) {
  pdl_enter();
  extern __shared__ __align__(16) unsigned char smem[];
  const int pad = ((n + 63) >> 6) << 6;
  int8_t* codes = reinterpret_cast<int8_t*>(smem);
  const int row = blockIdx.x;
  const float* xr = x + static_cast<size_t>(row) * n;
  const float sc = fmaxf(amax_in[row] / 127.0f, act_eps);
  const float rscale = 1.0f / sc;
  for (int i = threadIdx.x; i < pad; i += kThreads) {
    int q = 0;
    if (i < n) {
      const float v = xr[i];
      bool nr = false;
      q = quant_code_fast(v, rscale, nr);
      if (nr) q = static_cast<int>(rintf(v / sc));
    }
    codes[i] = static_cast<int8_t>(q);
  }
  __syncthreads();
  for (int k = threadIdx.x; k < (ldq >> 4); k += kThreads) {
    uint32_t o[4];
#pragma unroll
    for (int f = 0; f < 4; ++f) {
      uint32_t w = 0u;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int i = (k << 4) + 4 * b + f;
        w |= (i < n ? static_cast<uint32_t>(static_cast<uint8_t>(codes[i])) : 0u) << (8 * b);
      }
      o[f] = w;
    }
    *reinterpret_cast<uint4*>(q8 + q8_chunk_offset(row, k, ldq)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if (threadIdx.x == 0) scale[row] = sc;
}

}  // namespace ivb

extern "C" {

int32_t ivb_quantize_rows(const float* x, int32_t rows, int32_t n, const float* norm_weight, float norm_eps,
                          float norm_clip, float act_eps, int8_t* q8, int32_t ldq, float* scale, int32_t* gsum,
                          void* stream) {
  using namespace ivb;
  if (x == nullptr || q8 == nullptr || scale == nullptr) return fail(IVB_EINVAL, "ivb_quantize_rows: null argument");
  if (rows < 0 || n <= 0 || ldq < (n + 127) / 128 * 128 || (ldq & 127) || (reinterpret_cast<uintptr_t>(q8) & 15))
    return fail(IVB_EINVAL, "ivb_quantize_rows: bad shape (rows %d, n %d, ldq %d)", rows, n, ldq);
  if (rows == 0) return IVB_OK;
  const size_t pad = static_cast<size_t>((n + 63) / 64) * 64;
  const size_t smem = pad * 4 + pad + 64 * 4;
  if (smem > 200 * 1024) return fail(IVB_EINVAL, "ivb_quantize_rows: n %d too large", n);
  IVB_CUDA(cudaFuncSetAttribute(quantize_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  IVB_CUDA(launch_pdl(quantize_rows_kernel, dim3(rows), dim3(kThreads), smem, static_cast<cudaStream_t>(stream), x, n, norm_weight, norm_eps, norm_clip,
                                                                                   act_eps, q8, ldq, scale, gsum));
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

}  // extern "C"

namespace ivb {
namespace {
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}
}  // namespace
}  // namespace ivb

extern "C" {

}  // extern "C"

namespace ivb {
namespace {
// Multiprocessor count of device `dev`, looked up once per device.
cudaError_t sm_count(int dev, int* out) {
  static std::mutex lock;
  static int table[64] = {};
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> guard(lock);
  if (table[dev] == 0) {
    const cudaError_t rc = cudaDeviceGetAttribute(&table[dev], cudaDevAttrMultiProcessorCount, dev);
    if (rc != cudaSuccess) return rc;
  }
  *out = table[dev];
  return cudaSuccess;
}

int32_t gemm_scratch(int dev, float** out) {
  static std::mutex lock;
  static float* table[64] = {};
  if (dev < 0 || dev >= 64) return fail(IVB_EINVAL, "ivb_ternary_gemm: device %d out of range", dev);
  std::lock_guard<std::mutex> guard(lock);
  if (table[dev] == nullptr) {
    void* p = nullptr;
    IVB_CUDA(cudaGetSymbolAddress(&p, g_gemm_partial));  // once per device
    table[dev] = static_cast<float*>(p);
  }
  *out = table[dev];
  return IVB_OK;
}
}  // namespace
}  // namespace ivb

extern "C" {

int32_t ivb_ternary_gemm(const IvbTernary* m, const int8_t* q8, int32_t ldq, const float* act_scale, int32_t rows_t,
                         int32_t epilogue, float* out, int32_t ldo, uint32_t* error, void* stream) {
  using namespace ivb;
  int dev = 0;
  IVB_CUDA(cudaGetDevice(&dev));
  float* partial = nullptr;
  if (int32_t rc = gemm_scratch(dev, &partial)) return rc;
  return ternary_gemm_into(m, q8, ldq, act_scale, rows_t, epilogue, out, ldo, error, partial, kGemmPartialFloats, stream);
}

}  // extern "C"

int32_t ivb::ternary_gemm_into(const IvbTernary* m, const int8_t* q8, int32_t ldq, const float* act_scale, int32_t rows_t,
                               int32_t epilogue, float* out, int32_t ldo, uint32_t* error, float* partial, size_t partial_floats,
                               void* stream) {
  using namespace ivb;
  if (m == nullptr || q8 == nullptr || act_scale == nullptr || out == nullptr || error == nullptr)
    return fail(IVB_EINVAL, "ivb_ternary_gemm: null argument");
  if (int32_t rc = check_ternary(*m, "ivb_ternary_gemm")) return rc;
  if (epilogue < IVB_EPI_STORE || epilogue > IVB_EPI_SILU_PAIR) return fail(IVB_EINVAL, "ivb_ternary_gemm: bad epilogue");
  if (epilogue == IVB_EPI_SILU_PAIR && (m->rows & 1)) return fail(IVB_EINVAL, "ivb_ternary_gemm: silu pairs need an even row count");
  if (rows_t < 0 || ldq < (m->in_features + 127) / 128 * 128 || (ldq & 127) || (reinterpret_cast<uintptr_t>(q8) & 15))
    return fail(IVB_EINVAL, "ivb_ternary_gemm: bad activation layout (ldq %d)", ldq);
  if (ldo < (epilogue == IVB_EPI_SILU_PAIR ? m->rows / 2 : m->rows)) return fail(IVB_EINVAL, "ivb_ternary_gemm: ldo too small");
  if (rows_t == 0) return IVB_OK;
  if (!device_is_sm100()) return fail(IVB_EUNSUPPORTED, "ivb_ternary_gemm: needs an sm_100 device");
  const int groups = (m->in_features + 127) / 128;
  constexpr size_t kSmemCap = 227 * 1024 - 2048;  // dynamic shared memory beside the static barriers
  const size_t smem = static_cast<size_t>(kGemmStages) * kGemmTile + kPackSlots * kPackSlot + 1024;
  static_assert(static_cast<size_t>(kGemmStages) * kGemmTile + kPackSlots * kPackSlot + 1024 <= kSmemCap,
                "the GEMM's rings exceed shared memory");
  IVB_CUDA(cudaFuncSetAttribute(ternary_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (encode == nullptr) return fail(IVB_EUNSUPPORTED, "ivb_ternary_gemm: cuTensorMapEncodeTiled is unavailable");
  CUtensorMap wmap;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(m->row_bytes), static_cast<cuuint64_t>(m->rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(m->row_bytes)};
  const cuuint32_t box[2] = {32, kGemmRows}, estride[2] = {1, 1};
  if (encode(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<unsigned char*>(m->packed), dims, strides, box, estride,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return fail(IVB_EINVAL, "ivb_ternary_gemm: cannot describe the packed weights to the TMA engine");
  // split-K when the row and token tiles leave most SMs idle (decode-sized token counts): at least four
  // groups per split, at most 8 splits, the partials within the caller's scratch
  const int row_tiles = (m->rows + kGemmRows - 1) / kGemmRows, tok_tiles = (rows_t + kGemmTok - 1) / kGemmTok;
  int splits = 1;
  if (partial != nullptr && groups >= 8 && row_tiles * tok_tiles < 96) {
    splits = std::min({groups / 4, std::max(1, 148 / (row_tiles * tok_tiles)), 8});
    while (splits > 1 && static_cast<size_t>(splits) * rows_t * m->rows > partial_floats) --splits;
  }
  const int g_per = (groups + splits - 1) / splits;
  splits = (groups + g_per - 1) / g_per;
  if (splits == 1) partial = nullptr;
  const int units = row_tiles * tok_tiles * splits;
  int dev = 0, sms = 0;
  IVB_CUDA(cudaGetDevice(&dev));
  IVB_CUDA(sm_count(dev, &sms));
  const dim3 grid(std::min(units, sms));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // programmatic dependent launch: the kernel's set-up overlaps the tail of the previous kernel on the
  // stream (the kernel waits for that grid with griddepcontrol.wait before reading its outputs)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const IvbTernary mv = *m;
  IVB_CUDA(cudaLaunchKernelEx(&cfg, ternary_gemm_kernel, wmap, mv, q8, ldq, act_scale, static_cast<int>(rows_t), static_cast<int>(epilogue),
                              out, static_cast<int>(ldo), g_per, row_tiles, tok_tiles, units, partial, 2000000000ull, error));
  if (splits > 1) {
    const int per_row = epilogue == IVB_EPI_SILU_PAIR ? m->rows / 2 : m->rows;
    const int n = rows_t * per_row;
    IVB_CUDA(launch_pdl(gemm_splitk_reduce_kernel, dim3((n + 255) / 256), dim3(256), 0, s, partial, splits, rows_t, m->rows, act_scale, m->bias, epilogue,
                                                            out, ldo));
    IVB_CUDA(cudaGetLastError());
  }
  return IVB_OK;
}

extern "C" {

int32_t ivb_rows_amax(const float* x, int32_t rows, int32_t n, float* amax, void* stream) {
  using namespace ivb;
  if (x == nullptr || amax == nullptr || rows < 0 || n <= 0) return fail(IVB_EINVAL, "ivb_rows_amax: bad argument");
  if (rows == 0) return IVB_OK;
  IVB_CUDA(launch_pdl(rows_amax_kernel, dim3(rows), dim3(kThreads), 0, static_cast<cudaStream_t>(stream), x, n, amax));
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

int32_t ivb_quantize_rows_amax(const float* x, int32_t rows, int32_t n, const float* amax, float act_eps, int8_t* q8,
                               int32_t ldq, float* scale, void* stream) {
  using namespace ivb;
  if (x == nullptr || amax == nullptr || q8 == nullptr || scale == nullptr) return fail(IVB_EINVAL, "ivb_quantize_rows_amax: null argument");
  if (rows < 0 || n <= 0 || ldq < (n + 127) / 128 * 128 || (ldq & 127) || (reinterpret_cast<uintptr_t>(q8) & 15))
    return fail(IVB_EINVAL, "ivb_quantize_rows_amax: bad shape (rows %d, n %d, ldq %d)", rows, n, ldq);
  if (rows == 0) return IVB_OK;
  const size_t smem = static_cast<size_t>((n + 63) / 64) * 64 + 64;
  if (smem > 200 * 1024) return fail(IVB_EINVAL, "ivb_quantize_rows_amax: n %d too large", n);
  IVB_CUDA(cudaFuncSetAttribute(quantize_rows_amax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  IVB_CUDA(launch_pdl(quantize_rows_amax_kernel, dim3(rows), dim3(kThreads), smem, static_cast<cudaStream_t>(stream), x, n, amax, act_eps, q8, ldq, scale));
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

}  // extern "C"
