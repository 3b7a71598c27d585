// Prefill ternary GEMM of libivonar_b200.so on the 5th-generation tensor cores (tcgen05, kind::i8).
//
// out[t][r] = epilogue(act_scale[t] * sum_g s[r][g] * (sum_{k in g} code[r][k] * q8[t][k] - gsum[t][g]) + bias[r])
// for T token rows at once. codes are the 2-bit weights as unsigned bytes 0..2 (= ternary + 1), so the
// per-group integer dot is exact in the int32 accumulator and the -1 offset is the group sum of the
// activations. Reference: kernels/ternary.cu:688-765 gemm_tile_body (per-token int8 tiles, dp4a).
//
// One CTA computes a 128-token x 128-row tile; per 128-input scale group it stages the activations
// (already in the GEMM layout) and the unpacked weight codes in shared memory as K-major core matrices,
// one thread issues four 128x128x32 int8 MMAs into a TMEM accumulator, and the four warps read it back
// (tcgen05.ld), subtract the group sum, scale by the fp16 group scale and accumulate in fp32 registers.
#include <cuda_runtime.h>

#include "ivb_common.h"
#include "ivb_cluster.cuh"

namespace ivb {

constexpr int kGemmM = 128;          // tokens per tile (TMEM lanes)
constexpr int kGemmN = 128;          // weight rows per tile (TMEM columns)
constexpr int kGemmThreads = 128;    // four warps: warp w owns TMEM lanes 32w..32w+31
constexpr int kGemmTile = 16384;     // bytes of one 128 x 128 int8 operand tile

// Position of input i inside the GEMM activation layout: each 16-input block is a 4 x 4 byte transpose
// (byte 4f + b holds input 4b + f), which matches the codes a packed weight word yields by masking
// (w >> 2f) & 0x03030303 for f = 0..3.
__host__ __device__ __forceinline__ int gemm_slot(int i) { return (i & ~15) + ((i & 3) << 2) + ((i >> 2) & 3); }

// One 16-byte chunk (c) of row r in a K-major core-matrix tile: core matrices of 8 rows x 16 bytes,
// 8 chunks (128 inputs) per row group. LBO (next K chunk) = 128 B, SBO (next 8-row group) = 1024 B.
__device__ __forceinline__ int tile_off(int r, int c) { return (((r >> 3) << 3) + c) * 128 + ((r & 7) << 4); }

__device__ __forceinline__ uint64_t smem_desc(unsigned addr) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(128 >> 4) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46);
}

// kind::i8 instruction descriptor: D s32, A s8 (activations), B u8 (codes), both K-major, M 128, N 128.
constexpr uint32_t kGemmIdesc = (2u << 4) | (1u << 7) | (0u << 10) | (static_cast<uint32_t>(kGemmN >> 3) << 17) |
                                (static_cast<uint32_t>(kGemmM >> 4) << 24);

__device__ __forceinline__ void umma_i8(unsigned tmem_d, uint64_t da, uint64_t db, uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
}
__device__ __forceinline__ void umma_commit(unsigned long long* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(unsigned taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Grid (row tiles, token tiles). q8 [T][ldq] int8 in gemm_slot order, gsum [T][groups], act_scale [T].
__global__ void __launch_bounds__(kGemmThreads, 1) ternary_gemm_kernel(const IvbTernary m, const int8_t* __restrict__ q8,
                                                                       int ldq, const float* __restrict__ act_scale,
                                                                       const int32_t* __restrict__ gsum, int T,
                                                                       int epilogue, float* out, int ldo,
                                                                       unsigned long long timeout_ns, unsigned* error) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      smem_raw + ((1024u - (static_cast<unsigned>(__cvta_generic_to_shared(smem_raw)) & 1023u)) & 1023u);
  unsigned char* tile_a = smem;                    // [128 tokens][128] int8, core-matrix layout
  unsigned char* tile_b = smem + kGemmTile;        // [128 rows][128] codes
  float* scl = reinterpret_cast<float*>(smem + 2 * kGemmTile);  // [128] group scales of the tile's rows
  __shared__ __align__(8) unsigned long long mma_bar;
  __shared__ unsigned tmem_base;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int r0 = blockIdx.x * kGemmN, t0 = blockIdx.y * kGemmM;
  const int groups = (m.in_features + 127) >> 7;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(kGemmN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    mbar_init(&mma_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = tmem_base;
  const int t = t0 + tid;                 // the token row this thread drains (TMEM lane tid)
  const bool t_ok = t < T;
  float acc[kGemmN];
#pragma unroll
  for (int n = 0; n < kGemmN; ++n) acc[n] = 0.0f;
  unsigned parity = 0;
  bool late = false;
  for (int g = 0; g < groups && !late; ++g) {
    // stage A: this thread's token row, eight 16-byte chunks of group g
    {
      const uint4* src = reinterpret_cast<const uint4*>(q8 + static_cast<size_t>(t_ok ? t : 0) * ldq + (g << 7));
      const int kin = min(128, m.in_features - (g << 7));
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (t_ok && (c << 4) < kin) v = __ldg(src + c);
        *reinterpret_cast<uint4*>(tile_a + tile_off(tid, c)) = v;
      }
    }
    // stage B: this thread's weight row, eight packed words -> eight 16-byte code chunks
    {
      const int r = r0 + tid;
      const bool r_ok = r < m.rows;
      const uint32_t* src = reinterpret_cast<const uint32_t*>(m.packed + static_cast<size_t>(r_ok ? r : 0) * m.row_bytes) + (g << 3);
      const int words = min(8, (m.row_bytes >> 2) - (g << 3));
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint32_t w = (r_ok && c < words) ? __ldg(src + c) : 0u;
        uint4 v;
        v.x = w & 0x03030303u;
        v.y = (w >> 2) & 0x03030303u;
        v.z = (w >> 4) & 0x03030303u;
        v.w = (w >> 6) & 0x03030303u;
        *reinterpret_cast<uint4*>(tile_b + tile_off(tid, c)) = v;
      }
      scl[tid] = r_ok ? h2f(__ldg(m.scales + static_cast<size_t>(r) * m.scale_stride + g)) : 0.0f;
    }
    const float gs = t_ok ? static_cast<float>(__ldg(gsum + static_cast<size_t>(t) * groups + g)) : 0.0f;
    fence_proxy_async();  // the staged tiles, before the tensor core reads them
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const unsigned a = smem_addr(tile_a), b = smem_addr(tile_b);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) umma_i8(tmem, smem_desc(a + kk * 256), smem_desc(b + kk * 256), kGemmIdesc, kk > 0);
      umma_commit(&mma_bar);
    }
    // wait for the four MMAs (bounded), then drain this thread's lane
    late = !mbar_wait_bounded(&mma_bar, parity, timeout_ns);
    late = __syncthreads_or(late);
    parity ^= 1u;
    if (late) break;
    tc_fence_after();
    const unsigned lane_addr = tmem + (static_cast<unsigned>(warp * 32) << 16);
#pragma unroll
    for (int cb = 0; cb < kGemmN / 32; ++cb) {
      uint32_t d[32];
      tmem_ld32(lane_addr + cb * 32, d);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int n = cb * 32 + j;
        acc[n] = fmaf(static_cast<float>(static_cast<int>(d[j])) - gs, scl[n], acc[n]);
      }
    }
    tc_fence_before();
    __syncthreads();  // tiles and TMEM are rewritten by the next group
  }
  if (late) {
    if (tid == 0) atomicCAS(error, 0u, static_cast<unsigned>(IVB_ETIMEOUT));
  } else if (t_ok) {
    const float s = __ldg(act_scale + t);
    float* orow = out + static_cast<size_t>(t) * ldo;
    if (epilogue == IVB_EPI_SILU_PAIR) {
#pragma unroll
      for (int p2 = 0; p2 < kGemmN / 2; ++p2) {
        const int r = r0 + 2 * p2;
        if (r + 1 < m.rows) {
          float g = acc[2 * p2] * s, u = acc[2 * p2 + 1] * s;
          if (m.bias != nullptr) {
            g += __ldg(m.bias + r);
            u += __ldg(m.bias + r + 1);
          }
          orow[r >> 1] = silu_f(g) * u;
        }
      }
    } else {
#pragma unroll
      for (int n = 0; n < kGemmN; ++n) {
        const int r = r0 + n;
        if (r < m.rows) {
          float v = acc[n] * s;
          if (m.bias != nullptr) v += __ldg(m.bias + r);
          orow[r] = epilogue == IVB_EPI_RESIDUAL ? orow[r] + v : v;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kGemmN));
}

// One CTA per token row: the canonical quantiser (RMSNorm optional), codes written in gemm_slot order,
// per-128-group sums of the codes.
__global__ void __launch_bounds__(kThreads) quantize_rows_kernel(const float* x, int n, const float* norm_w, float norm_eps,
                                                                 float clip, float act_eps, int8_t* q8, int ldq,
                                                                 float* scale, int32_t* gsum) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int pad = ((n + 63) >> 6) << 6;
  float* xv = reinterpret_cast<float*>(smem);
  int8_t* codes = reinterpret_cast<int8_t*>(xv + pad);
  float* red = reinterpret_cast<float*>(codes + pad);
  const int row = blockIdx.x;
  load_vector(x + static_cast<size_t>(row) * n, n, xv);
  __syncthreads();
  const float s = quantize_block(xv, n, norm_w, norm_eps, clip, act_eps, codes, false, nullptr, red);
  int8_t* qrow = q8 + static_cast<size_t>(row) * ldq;
  const int groups = (n + 127) >> 7;
  for (int i = threadIdx.x; i < ldq; i += kThreads) qrow[gemm_slot(i)] = i < n ? codes[i] : 0;
  // group sums: one warp per group, exact integers
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int g = warp; g < groups; g += kWarps) {
    int sum = 0;
    for (int i = (g << 7) + lane; i < min(n, (g + 1) << 7); i += 32) sum += codes[i];
    sum = __reduce_add_sync(kFull, sum);
    if (lane == 0) gsum[static_cast<size_t>(row) * groups + g] = sum;
  }
  if (threadIdx.x == 0) scale[row] = s;
}

}  // namespace ivb

extern "C" {

int32_t ivb_quantize_rows(const float* x, int32_t rows, int32_t n, const float* norm_weight, float norm_eps,
                          float norm_clip, float act_eps, int8_t* q8, int32_t ldq, float* scale, int32_t* gsum,
                          void* stream) {
  using namespace ivb;
  if (x == nullptr || q8 == nullptr || scale == nullptr || gsum == nullptr)
    return fail(IVB_EINVAL, "ivb_quantize_rows: null argument");
  if (rows < 0 || n <= 0 || ldq < (n + 127) / 128 * 128 || (ldq & 15))
    return fail(IVB_EINVAL, "ivb_quantize_rows: bad shape (rows %d, n %d, ldq %d)", rows, n, ldq);
  if (rows == 0) return IVB_OK;
  const size_t pad = static_cast<size_t>((n + 63) / 64) * 64;
  const size_t smem = pad * 4 + pad + 64 * 4;
  if (smem > 200 * 1024) return fail(IVB_EINVAL, "ivb_quantize_rows: n %d too large", n);
  IVB_CUDA(cudaFuncSetAttribute(quantize_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  quantize_rows_kernel<<<rows, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(x, n, norm_weight, norm_eps, norm_clip,
                                                                                   act_eps, q8, ldq, scale, gsum);
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

int32_t ivb_ternary_gemm(const IvbTernary* m, const int8_t* q8, int32_t ldq, const float* act_scale, const int32_t* gsum,
                         int32_t rows_t, int32_t epilogue, float* out, int32_t ldo, uint32_t* error, void* stream) {
  using namespace ivb;
  if (m == nullptr || q8 == nullptr || act_scale == nullptr || gsum == nullptr || out == nullptr || error == nullptr)
    return fail(IVB_EINVAL, "ivb_ternary_gemm: null argument");
  if (int32_t rc = check_ternary(*m, "ivb_ternary_gemm")) return rc;
  if (epilogue < IVB_EPI_STORE || epilogue > IVB_EPI_SILU_PAIR) return fail(IVB_EINVAL, "ivb_ternary_gemm: bad epilogue");
  if (epilogue == IVB_EPI_SILU_PAIR && (m->rows & 1)) return fail(IVB_EINVAL, "ivb_ternary_gemm: silu pairs need an even row count");
  if (rows_t < 0 || ldq < (m->in_features + 127) / 128 * 128 || (ldq & 15) || (reinterpret_cast<uintptr_t>(q8) & 15))
    return fail(IVB_EINVAL, "ivb_ternary_gemm: bad activation layout (ldq %d)", ldq);
  if (ldo < (epilogue == IVB_EPI_SILU_PAIR ? m->rows / 2 : m->rows)) return fail(IVB_EINVAL, "ivb_ternary_gemm: ldo too small");
  if (rows_t == 0) return IVB_OK;
  if (!device_is_sm100()) return fail(IVB_EUNSUPPORTED, "ivb_ternary_gemm: needs an sm_100 device");
  const size_t smem = 2 * kGemmTile + kGemmN * 4 + 1024;
  IVB_CUDA(cudaFuncSetAttribute(ternary_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  const dim3 grid((m->rows + kGemmN - 1) / kGemmN, (rows_t + kGemmM - 1) / kGemmM);
  ternary_gemm_kernel<<<grid, kGemmThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      *m, q8, ldq, act_scale, gsum, rows_t, epilogue, out, ldo, 2000000000ull, error);
  IVB_CUDA(cudaGetLastError());
  return IVB_OK;
}

}  // extern "C"
