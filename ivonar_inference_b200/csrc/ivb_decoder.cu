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
#include <vector>

#include "ivb_common.h"
#include "ivb_device.cuh"

size_t ivb_sample_smem_bytes(int vocab);
size_t ivb_gemv_smem_bytes(int n);
int ivb_lpr_log(int in_features);

namespace ivb {

enum PhaseKind : int32_t { PH_GEMV = 0, PH_SSM = 1, PH_ATTN = 2, PH_HEAD = 3, PH_SAMPLE = 4 };

struct Phase {
  int32_t kind;
  int32_t epilogue;
  int32_t layer;
  int32_t embed_input;  // input vector = embedding row of the current token
  IvbTernary mat;
  const float* in_vec;
  const float* norm_w;
  float norm_eps;
  int32_t rows_per_cta;
  float* out_vec;
  int32_t lpr_log;
  int32_t pad_;
};

struct Dims {
  int32_t vocab, hidden, heads, head_dim, state_dim, latent, rope, nope, dense, max_len, max_top_k, mixer_width;
  float act_eps, clip;
};

struct RunParams {
  const Phase* prog;
  int32_t n_phases;
  int32_t steps;
  const IvbLayerDesc* layers;
  Dims dims;
  IvbTernary head;
  float* residual;
  float* mixer_in;
  float* ybuf;
  float* ffn_mid;
  float* logits;
  int64_t* token;
  int64_t* position;
  uint8_t* seen;
  int64_t* history;
  const float* sampling;
  const int64_t* top_k;
  uint64_t* rng;
  unsigned* counter;
  unsigned* error;
  const int64_t* feed;
  unsigned long long timeout_ns;
  int32_t history_len;
  int32_t flags;
};

struct SmemPlan {
  size_t gemv, attn, sample, total;
};

__device__ __forceinline__ void carve_sample(unsigned char* smem, int vocab, SampleSmem& sm) {
  sm.keys = reinterpret_cast<unsigned*>(smem);
  sm.hist = sm.keys + vocab;
  sm.ckey = sm.hist + kWarps * 256;
  sm.cidx = reinterpret_cast<int*>(sm.ckey + kMaxTopK);
  sm.cprob = reinterpret_cast<float*>(sm.cidx + kMaxTopK);
  sm.misc = reinterpret_cast<int*>(sm.cprob + kMaxTopK);
  sm.red = reinterpret_cast<float*>(sm.misc + 16);
}

__device__ __forceinline__ void carve_attn(unsigned char* smem, const Dims& D, AttnSmem& sm) {
  const int lpad = ((D.latent + 63) >> 6) << 6;
  float* f = reinterpret_cast<float*>(smem);
  sm.xv = f;
  f += lpad;
  sm.qa = f;
  f += lpad;
  sm.qr = f;
  f += D.rope;
  sm.kr = f;
  f += D.rope;
  sm.qn = f;
  f += D.nope;
  sm.red = f;
  f += 64;
  sm.part = f;
  f += kWarps * (D.latent + 2);
  sm.ql = reinterpret_cast<int8_t*>(f);
}

__host__ __device__ inline size_t attn_smem_bytes(int latent, int rope, int nope) {
  const size_t lpad = static_cast<size_t>((latent + 63) / 64) * 64;
  return (lpad * 2 + rope * 2 + nope + 64 + kWarps * (latent + 2)) * 4 + lpad + 16;
}

__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ RunParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int bflag;
  const int cta = blockIdx.x, G = gridDim.x, tid = threadIdx.x;
  const Dims& D = p.dims;
  if (p.flags & IVB_RUN_SAMPLE_ONLY) {
    if (cta == 0) {
      SampleSmem sm;
      carve_sample(smem, D.vocab, sm);
      sample_block(p.logits, p.seen, D.vocab, p.sampling, p.top_k, D.max_top_k, p.rng, p.token, nullptr, sm);
    }
    return;
  }
  const Sync sync{p.counter, p.error, p.timeout_ns};
  const bool sample = (p.flags & IVB_RUN_SAMPLE) != 0;
  unsigned bars = 0;
  uint4 pf[kPrefetch];
  float pfs[kPrefetch];
  int pf_for = -1;
  const int n = p.n_phases;  // [5 per layer] + HEAD + SAMPLE
  for (int step = 0; step < p.steps; ++step) {
    const long long tok = p.feed != nullptr ? ldcg_i64(p.feed + step) : ldcg_i64(p.token);
    const long long pos = ldcg_i64(p.position);
    if (pos < 0 || pos >= D.max_len) {
      if (cta == 0 && tid == 0) atomicCAS(p.error, 0u, static_cast<unsigned>(IVB_ECAPACITY));
      return;
    }
    if (tok < 0 || tok >= D.vocab) {
      if (cta == 0 && tid == 0) atomicCAS(p.error, 0u, static_cast<unsigned>(IVB_EINVAL));
      return;
    }
    const bool head = sample || (p.flags & IVB_RUN_HEAD_ALL) != 0 || step == p.steps - 1;
    const int last = sample ? n - 1 : (head ? n - 2 : n - 3);
    for (int pi = 0; pi <= last; ++pi) {
      const Phase ph = p.prog[pi];
      if (ph.kind == PH_GEMV || ph.kind == PH_HEAD) {
        const GemvGeom g = gemv_geom(ph.mat, ph.rows_per_cta, ph.lpr_log, cta);
        if (pf_for != pi) gemv_prefetch(ph.mat, g, pf, pfs);
        const int nin = ph.mat.in_features;
        const int pad = ((nin + 63) >> 6) << 6;
        float* xv = reinterpret_cast<float*>(smem);
        int8_t* act = reinterpret_cast<int8_t*>(xv + pad);
        int* xs = reinterpret_cast<int*>(act + pad);
        float* red = reinterpret_cast<float*>(xs + (pad >> 6));
        float* res = red + 64;
        if (ph.embed_input) {
          const uint8_t* erow = p.head.packed + static_cast<size_t>(tok) * p.head.row_bytes;
          const uint16_t* srow = p.head.scales + static_cast<size_t>(tok) * p.head.scale_stride;
          const int per = (nin + G - 1) / G;
          for (int i = tid; i < nin; i += kThreads) {
            const int code = (__ldg(erow + (i >> 2)) >> ((i & 3) << 1)) & 3;
            const float v = static_cast<float>(code - 1) * h2f(__ldg(srow + (i >> 7)));
            xv[i] = v;
            if (i >= cta * per && i < (cta + 1) * per) p.residual[i] = v;
          }
        } else {
          for (int i = tid; i < nin; i += kThreads) xv[i] = ldcg_f(ph.in_vec + i);
        }
        __syncthreads();
        if (g.r0 < g.r1) {
          const float s = quantize_block(xv, nin, ph.norm_w, ph.norm_eps, D.clip, D.act_eps, act, true, xs, red);
          gemv_rows(ph.mat, g, act, xs, s, ph.epilogue, ph.out_vec, pf, pfs, res);
        }
      } else if (ph.kind == PH_SSM) {
        const IvbLayerDesc L = p.layers[ph.layer];
        const int per = (D.hidden + G - 1) / G;
        const int c0 = min(D.hidden, cta * per), c1 = min(D.hidden, c0 + per);
        ssm_channels(L, D.hidden, D.heads, D.head_dim, D.state_dim, p.mixer_in, p.ybuf, c0, c1);
      } else if (ph.kind == PH_ATTN) {
        const IvbLayerDesc L = p.layers[ph.layer];
        AttnSmem sm;
        carve_attn(smem, D, sm);
        for (int h = cta; h < D.heads; h += G)
          attention_head(L, D.hidden, D.heads, D.head_dim, D.nope, D.rope, D.latent, D.act_eps, p.mixer_in, p.ybuf, h,
                         static_cast<int>(pos), sm);
      } else if (ph.kind == PH_SAMPLE) {
        if (cta == 0) {
          SampleSmem sm;
          carve_sample(smem, D.vocab, sm);
          int64_t* hist = (p.history != nullptr && step < p.history_len) ? p.history + step : nullptr;
          sample_block(p.logits, p.seen, D.vocab, p.sampling, p.top_k, D.max_top_k, p.rng, p.token, hist, sm);
        }
      }
      if (pi == last && cta == 0 && tid == 0) p.position[0] = pos + 1;
      // load the first weight chunks of the next GEMV slice before waiting
      int nxt = pi < last ? pi + 1 : (step + 1 < p.steps ? 0 : -1);
      pf_for = -1;
      if (nxt >= 0) {
        const Phase& q = p.prog[nxt];
        if (q.kind == PH_GEMV || q.kind == PH_HEAD) {
          const GemvGeom g = gemv_geom(q.mat, q.rows_per_cta, q.lpr_log, cta);
          gemv_prefetch(q.mat, g, pf, pfs);
          pf_for = nxt;
        }
      }
      if (!grid_barrier(sync, (++bars) * static_cast<unsigned>(G), &bflag)) return;
    }
  }
}

}  // namespace ivb

// ------------------------------------------------------------------------------------------------
// host plan
// ------------------------------------------------------------------------------------------------
struct IvbDecoder {
  IvbModelDesc desc;
  std::vector<IvbLayerDesc> layers;
  std::vector<ivb::Phase> prog;
  ivb::Dims dims;
  int32_t ctas;
  size_t smem;
  size_t off_prog, off_layers, off_sync, off_residual, off_mixer, off_y, off_ffn, total;
  unsigned char* ws;
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
        L.down.rows != d.hidden || L.down.in_features != d.dense || L.gate_up.in_features != d.hidden)
      return fail(IVB_EINVAL, "layer %d: projection shapes do not match the model dimensions", i);
    if (!L.mixer_norm || !L.ffn_norm) return fail(IVB_EINVAL, "layer %d: null norm weight", i);
    if (L.kind == IVB_MAMBA) {
      if (L.entry.rows != 2 * d.hidden + 3 * d.heads * d.state_dim || L.out.in_features != d.hidden)
        return fail(IVB_EINVAL, "layer %d: mamba entry must be [2*hidden + 3*heads*state, hidden]", i);
      if (!L.decay || !L.theta || !L.skip || !L.conv_weight || !L.conv_bias || !L.ssm_state || !L.prev_force ||
          !L.conv_state || L.conv_taps < 1)
        return fail(IVB_EINVAL, "layer %d: missing recurrent constants or state", i);
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
    } else {
      return fail(IVB_EINVAL, "layer %d: unknown kind %d", i, L.kind);
    }
  }
  return IVB_OK;
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
  Dims& D = dec->dims;
  D.vocab = desc->vocab;
  D.hidden = desc->hidden;
  D.heads = desc->heads;
  D.head_dim = desc->head_dim;
  D.state_dim = desc->state_dim;
  D.latent = desc->latent_dim;
  D.rope = desc->rope_dim;
  D.nope = desc->nope_dim;
  D.dense = desc->dense;
  D.max_len = desc->max_len;
  D.max_top_k = desc->max_top_k;
  D.act_eps = desc->act_eps;
  D.clip = desc->norm_clip;
  int mixer_width = D.hidden;
  int widest = std::max(D.hidden, D.dense);
  bool any_mla = false;
  for (const IvbLayerDesc& L : dec->layers) {
    mixer_width = std::max(mixer_width, L.entry.rows);
    if (L.kind == IVB_MLA) any_mla = true;
  }
  D.mixer_width = mixer_width;
  int dev = 0, sms = 0;
  IVB_CUDA(cudaGetDevice(&dev));
  IVB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  if (ctas <= 0) ctas = sms;
  size_t smem = ivb_gemv_smem_bytes(widest);
  if (any_mla) smem = std::max(smem, attn_smem_bytes(D.latent, D.rope, D.nope));
  smem = std::max(smem, ivb_sample_smem_bytes(D.vocab));
  if (smem > 227 * 1024) {
    delete dec;
    return fail(IVB_EINVAL, "the decoder needs %zu bytes of shared memory per CTA (vocab too large?)", smem);
  }
  IVB_CUDA(cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  int per_sm = 0;
  IVB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_kernel, kThreads, smem));
  if (per_sm < 1 || ctas > per_sm * sms) {
    delete dec;
    return fail(IVB_EINVAL, "%d CTAs cannot be co-resident (%d per SM x %d SMs)", ctas, per_sm, sms);
  }
  dec->ctas = ctas;
  dec->smem = smem;
  size_t off = 0;
  const size_t n_phases = static_cast<size_t>(desc->num_layers) * 5 + 2;
  dec->off_prog = off;
  off = align_up(off + n_phases * sizeof(Phase), 256);
  dec->off_layers = off;
  off = align_up(off + dec->layers.size() * sizeof(IvbLayerDesc), 256);
  dec->off_sync = off;
  off = align_up(off + 256, 256);
  dec->off_residual = off;
  off = align_up(off + static_cast<size_t>(D.hidden) * 4, 256);
  dec->off_mixer = off;
  off = align_up(off + static_cast<size_t>(mixer_width) * 4, 256);
  dec->off_y = off;
  off = align_up(off + static_cast<size_t>(D.hidden) * 4, 256);
  dec->off_ffn = off;
  off = align_up(off + static_cast<size_t>(D.dense) * 4, 256);
  dec->total = off;
  dec->ws = nullptr;
  *out = dec;
  return IVB_OK;
}

void ivb_decoder_destroy(IvbDecoder* dec) { delete dec; }

uint64_t ivb_decoder_workspace_bytes(const IvbDecoder* dec) { return dec ? dec->total : 0; }

int32_t ivb_decoder_num_phases(const IvbDecoder* dec) {
  return dec ? static_cast<int32_t>(dec->layers.size() * 5 + 2) : 0;
}

int32_t ivb_decoder_ctas(const IvbDecoder* dec) { return dec ? dec->ctas : 0; }

int32_t ivb_decoder_bind(IvbDecoder* dec, void* workspace, void* stream) {
  using namespace ivb;
  if (dec == nullptr || workspace == nullptr) return fail(IVB_EINVAL, "ivb_decoder_bind: null argument");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return fail(IVB_EINVAL, "workspace must be 256-byte aligned");
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  dec->ws = ws;
  float* residual = reinterpret_cast<float*>(ws + dec->off_residual);
  float* mixer = reinterpret_cast<float*>(ws + dec->off_mixer);
  float* y = reinterpret_cast<float*>(ws + dec->off_y);
  float* ffn = reinterpret_cast<float*>(ws + dec->off_ffn);
  const int G = dec->ctas;
  auto gemv = [&](const IvbTernary& m, int epi, int layer, const float* in, const float* norm, float eps, float* out,
                  int kind) {
    Phase ph{};
    ph.kind = kind;
    ph.epilogue = epi;
    ph.layer = layer;
    ph.embed_input = 0;
    ph.mat = m;
    ph.in_vec = in;
    ph.norm_w = norm;
    ph.norm_eps = eps;
    int per = (m.rows + G - 1) / G;
    if (per & 1) ++per;
    ph.rows_per_cta = per;
    ph.out_vec = out;
    ph.lpr_log = ivb_lpr_log(m.in_features);
    return ph;
  };
  dec->prog.clear();
  for (int i = 0; i < static_cast<int>(dec->layers.size()); ++i) {
    const IvbLayerDesc& L = dec->layers[i];
    Phase entry = gemv(L.entry, IVB_EPI_STORE, i, residual, L.mixer_norm, L.mixer_norm_eps, mixer, PH_GEMV);
    entry.embed_input = i == 0 ? 1 : 0;
    dec->prog.push_back(entry);
    Phase mix{};
    mix.kind = L.kind == IVB_MAMBA ? PH_SSM : PH_ATTN;
    mix.layer = i;
    dec->prog.push_back(mix);
    dec->prog.push_back(gemv(L.out, IVB_EPI_RESIDUAL, i, y, nullptr, 0.0f, residual, PH_GEMV));
    dec->prog.push_back(gemv(L.gate_up, IVB_EPI_SILU_PAIR, i, residual, L.ffn_norm, L.ffn_norm_eps, ffn, PH_GEMV));
    dec->prog.push_back(gemv(L.down, IVB_EPI_RESIDUAL, i, ffn, nullptr, 0.0f, residual, PH_GEMV));
  }
  dec->prog.push_back(gemv(dec->desc.head, IVB_EPI_STORE, -1, residual, dec->desc.final_norm, dec->desc.final_norm_eps,
                           dec->desc.logits, PH_HEAD));
  Phase smp{};
  smp.kind = PH_SAMPLE;
  smp.layer = -1;
  dec->prog.push_back(smp);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  IVB_CUDA(cudaMemcpyAsync(ws + dec->off_prog, dec->prog.data(), dec->prog.size() * sizeof(Phase), cudaMemcpyHostToDevice, s));
  IVB_CUDA(cudaMemcpyAsync(ws + dec->off_layers, dec->layers.data(), dec->layers.size() * sizeof(IvbLayerDesc),
                           cudaMemcpyHostToDevice, s));
  IVB_CUDA(cudaMemsetAsync(ws + dec->off_sync, 0, 256, s));
  IVB_CUDA(cudaMemsetAsync(residual, 0, static_cast<size_t>(dec->dims.hidden) * 4, s));
  IVB_CUDA(cudaStreamSynchronize(s));
  return IVB_OK;
}

int32_t ivb_decoder_run(IvbDecoder* dec, int32_t steps, const int64_t* feed, int32_t flags, uint64_t timeout_ns,
                        void* stream) {
  using namespace ivb;
  if (dec == nullptr || dec->ws == nullptr) return fail(IVB_EINVAL, "ivb_decoder_run: decoder not bound");
  if (steps < 0) return fail(IVB_EINVAL, "ivb_decoder_run: negative step count");
  const bool sample_only = (flags & IVB_RUN_SAMPLE_ONLY) != 0;
  if (!sample_only && steps == 0) return IVB_OK;
  if (!sample_only && feed == nullptr && !(flags & IVB_RUN_SAMPLE))
    return fail(IVB_EINVAL, "ivb_decoder_run: without fed tokens every step must sample");
  const long long barriers = static_cast<long long>(steps) * static_cast<long long>(dec->prog.size()) * dec->ctas;
  if (barriers >= (1ll << 31)) return fail(IVB_EINVAL, "ivb_decoder_run: too many steps for one launch");
  RunParams p{};
  unsigned char* ws = dec->ws;
  p.prog = reinterpret_cast<const Phase*>(ws + dec->off_prog);
  p.n_phases = static_cast<int32_t>(dec->prog.size());
  p.steps = steps;
  p.layers = reinterpret_cast<const IvbLayerDesc*>(ws + dec->off_layers);
  p.dims = dec->dims;
  p.head = dec->desc.head;
  p.residual = reinterpret_cast<float*>(ws + dec->off_residual);
  p.mixer_in = reinterpret_cast<float*>(ws + dec->off_mixer);
  p.ybuf = reinterpret_cast<float*>(ws + dec->off_y);
  p.ffn_mid = reinterpret_cast<float*>(ws + dec->off_ffn);
  p.logits = dec->desc.logits;
  p.token = dec->desc.token;
  p.position = dec->desc.position;
  p.seen = dec->desc.seen;
  p.history = dec->desc.history;
  p.history_len = dec->desc.history_len;
  p.sampling = dec->desc.sampling;
  p.top_k = dec->desc.top_k;
  p.rng = dec->desc.rng;
  p.counter = reinterpret_cast<unsigned*>(ws + dec->off_sync);
  p.error = p.counter + 1;
  p.feed = feed;
  p.timeout_ns = timeout_ns == 0 ? 1000000000ull : timeout_ns;
  p.flags = flags;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  IVB_CUDA(cudaMemsetAsync(p.counter, 0, 2 * sizeof(unsigned), s));
  if (sample_only) {
    decode_kernel<<<1, kThreads, dec->smem, s>>>(p);
    IVB_CUDA(cudaGetLastError());
    return IVB_OK;
  }
  void* args[] = {&p};
  IVB_CUDA(cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(decode_kernel), dim3(dec->ctas), dim3(kThreads),
                                       args, dec->smem, s));
  return IVB_OK;
}

int32_t ivb_decoder_check(IvbDecoder* dec, void* stream) {
  using namespace ivb;
  if (dec == nullptr || dec->ws == nullptr) return fail(IVB_EINVAL, "ivb_decoder_check: decoder not bound");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  IVB_CUDA(cudaStreamSynchronize(s));
  unsigned word = 0;
  IVB_CUDA(cudaMemcpy(&word, dec->ws + dec->off_sync + sizeof(unsigned), sizeof(word), cudaMemcpyDeviceToHost));
  if (word == IVB_ECAPACITY) return fail(IVB_ECAPACITY, "the decoder has no free position left");
  if (word == IVB_EINVAL) return fail(IVB_EINVAL, "a token id is out of range for the vocabulary");
  if (word != 0) return fail(static_cast<int32_t>(word), "a bounded inter-CTA wait gave up (device error word %u)", word);
  return IVB_OK;
}

}  // extern "C"
