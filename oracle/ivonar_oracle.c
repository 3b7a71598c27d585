/*
 * ivonar_oracle.c — CPU restatement of the Ivonar token loop. TEST INFRASTRUCTURE ONLY.
 *
 * This is the checker for the sm_100a kernels in ivonar_inference_b200/csrc and the CPU baseline
 * timed beside them (bench.py cpu_baseline / --impl reference). Nothing in the product path loads it.
 * It restates the reference algorithm (LuisOezdem/ivonar-inference, src/ivonar_inference/...):
 *   - q2_g128 weight format                    quantization.py:13-32
 *   - activation quantiser + RMSNorm           kernels/ternary.cu:148-197, cpu_decoder.py:30-70
 *   - ternary x int8 GEMV (int per 64-chunk)   kernels/ternary.cu:241-258,302-354; cpu_decoder.py:73-125
 *   - recurrent step                           kernels/ternary.cu:421-482; cpu_decoder.py:137-183
 *   - latent attention step (fp32 K/V cache)   cpu_decoder.py:186-231; decoder.py:271-297
 *   - embedding row                            kernels/ternary.cu:411-419
 * and, where the reference leaves an order or a random source open, the canonical choices of the
 * B200 kernels (documented at each function): the 256-lane reduction order of the sum of squares,
 * the top-k tie order, the CDF scan order and the Philox4x32-10 uniform.
 * Pinned against vectors generated from the reference (tests/golden/make_golden.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_LANES 256
#define ORC_WARPS 8

static inline float h2f(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu;
  const uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal */
      int e = -1;
      uint32_t m = man;
      do {
        m <<= 1;
        ++e;
      } while ((m & 0x400u) == 0);
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3ffu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* Sum of squares in the kernels' order: lane t (of 256) accumulates x[t], x[t+256], ... with fmaf;
 * each warp of 32 lanes is reduced by an xor butterfly (offsets 16, 8, 4, 2, 1); the 8 warp totals
 * are added in order. */
static float canonical_sum_squares(const float* x, int n) {
  float lane[ORC_LANES];
  for (int t = 0; t < ORC_LANES; ++t) {
    float p = 0.0f;
    for (int i = t; i < n; i += ORC_LANES) p = fmaf(x[i], x[i], p);
    lane[t] = p;
  }
  float total = 0.0f;
  for (int w = 0; w < ORC_WARPS; ++w) {
    float v[32], nv[32];
    memcpy(v, lane + 32 * w, sizeof(v));
    for (int off = 16; off > 0; off >>= 1) {
      for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ off];
      memcpy(v, nv, sizeof(v));
    }
    total = (w == 0) ? v[0] : total + v[0];
  }
  return total;
}

/* Per-token int8 quantiser. norm_w != NULL: v = clamp(x * inv_rms, -clip, clip) * w with
 * inv_rms = 1 / sqrtf(ss / n + eps). scale = max(amax / 127, act_eps); q = rint(v / scale).
 * xsum (may be NULL): sums of q over 64-input chunks. Returns scale. */
float orc_quantize(const float* x, const float* norm_w, int n, float norm_eps, float clip, float act_eps, int8_t* q,
                   int32_t* xsum) {
  float* v = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
  if (norm_w) {
    const float ss = canonical_sum_squares(x, n);
    const float inv = 1.0f / sqrtf(ss / (float)n + norm_eps);
    for (int i = 0; i < n; ++i) {
      const float a = x[i] * inv;
      v[i] = fminf(fmaxf(a, -clip), clip) * norm_w[i];
    }
  } else {
    memcpy(v, x, sizeof(float) * (size_t)n);
  }
  float amax = 0.0f;
  for (int i = 0; i < n; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const float scale = fmaxf(amax / 127.0f, act_eps);
  for (int i = 0; i < n; ++i) q[i] = (int8_t)(int)rintf(v[i] / scale);
  if (xsum) {
    const int chunks = (n + 63) / 64;
    for (int u = 0; u < chunks; ++u) {
      int32_t s = 0;
      for (int i = 64 * u; i < 64 * u + 64 && i < n; ++i) s += q[i];
      xsum[u] = s;
    }
  }
  free(v);
  return scale;
}

static inline int code_at(const uint8_t* row, int i) { return (row[i >> 2] >> ((i & 3) * 2)) & 3; }

/* Exact integer core: dots[r * groups + g] = sum over inputs i of group g of (code - 1) * q8[i]. */
void orc_group_dots(const uint8_t* packed, int rows, int in, int row_bytes, const int8_t* q8, int32_t* dots,
                    int threads) {
  const int groups = (in + 127) / 128;
#pragma omp parallel for num_threads(threads > 0 ? threads : 1) schedule(static)
  for (int r = 0; r < rows; ++r) {
    const uint8_t* row = packed + (size_t)r * row_bytes;
    for (int g = 0; g < groups; ++g) {
      int32_t acc = 0;
      const int end = (g + 1) * 128 < in ? (g + 1) * 128 : in;
      for (int i = g * 128; i < end; ++i) acc += (code_at(row, i) - 1) * (int32_t)q8[i];
      dots[(size_t)r * groups + g] = acc;
    }
  }
}

/* out[r] = act_scale * sum over 64-chunks u of (float)(int dot of chunk u) * scale[r][u/2] + bias[r].
 * epilogue 0: store, 1: out[r] += result, 2: rows interleaved (2m gate, 2m+1 up): out[m] = silu(g)*u. */
void orc_gemv(const uint8_t* packed, const uint16_t* scales, int scale_stride, const float* bias, int rows, int in,
              int row_bytes, const int8_t* q8, float act_scale, float* out, int epilogue, int threads) {
  const int chunks = (in + 63) / 64;
  float* res = (float*)malloc(sizeof(float) * (size_t)rows);
#pragma omp parallel for num_threads(threads > 0 ? threads : 1) schedule(static)
  for (int r = 0; r < rows; ++r) {
    const uint8_t* row = packed + (size_t)r * row_bytes;
    const uint16_t* srow = scales + (size_t)r * scale_stride;
    float acc = 0.0f;
    for (int u = 0; u < chunks; ++u) {
      int32_t d = 0;
      const int end = 64 * u + 64 < in ? 64 * u + 64 : in;
      const uint8_t* bytes = row + 16 * u;
      int i = 64 * u;
      if (end - i == 64) {
        for (int b = 0; b < 16; ++b) {
          const int byte = bytes[b];
          const int8_t* qq = q8 + 64 * u + 4 * b;
          d += ((byte & 3) - 1) * qq[0] + (((byte >> 2) & 3) - 1) * qq[1] + (((byte >> 4) & 3) - 1) * qq[2] +
               (((byte >> 6) & 3) - 1) * qq[3];
        }
      } else {
        for (; i < end; ++i) d += (code_at(row, i) - 1) * (int32_t)q8[i];
      }
      acc = fmaf((float)d, h2f(srow[u >> 1]), acc);
    }
    float result = acc * act_scale;
    if (bias) result += bias[r];
    res[r] = result;
  }
  if (epilogue == 2) {
    for (int m = 0; m < rows / 2; ++m) {
      const float g = res[2 * m], u = res[2 * m + 1];
      out[m] = g / (1.0f + expf(-g)) * u;
    }
  } else if (epilogue == 1) {
    for (int r = 0; r < rows; ++r) out[r] += res[r];
  } else {
    for (int r = 0; r < rows; ++r) out[r] = res[r];
  }
  free(res);
}

/* Embedding row of the tied ternary head: (code - 1) * scale. */
void orc_embed(const uint8_t* packed, const uint16_t* scales, int scale_stride, int row_bytes, int hidden, int64_t token,
               float* out) {
  const uint8_t* row = packed + (size_t)token * row_bytes;
  const uint16_t* srow = scales + (size_t)token * scale_stride;
  for (int i = 0; i < hidden; ++i) out[i] = (float)(code_at(row, i) - 1) * h2f(srow[i >> 7]);
}

static inline float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

/* Recurrent step (reference ternary.cu:421-482): mixer_in = [value | gate | bc_dt]. */
void orc_ssm_step(const float* mixer_in, int hidden, int heads, int state_dim, int head_dim, int taps,
                  const float* conv_w, const float* conv_b, float* conv_state, const float* decay, const float* theta,
                  const float* skip, float* ssm_state, float* prev_force, float half_dt_min, float half_dt_range,
                  float* y) {
  for (int c = 0; c < hidden; ++c) {
    const int h = c / head_dim, d = c - h * head_dim;
    const float* w = conv_w + (size_t)c * taps;
    float* win = conv_state + (size_t)c * (taps - 1);
    const float incoming = mixer_in[c];
    float conv = conv_b[c];
    for (int k = 0; k < taps - 1; ++k) conv += w[k] * win[k];
    conv += w[taps - 1] * incoming;
    for (int k = 0; k + 1 < taps - 1; ++k) win[k] = win[k + 1];
    if (taps > 1) win[taps - 2] = incoming;
    const float value = conv / (1.0f + expf(-conv));
    const float* bcdt = mixer_in + 2 * hidden + h * 3 * state_dim;
    float total = 0.0f;
    for (int s = 0; s < state_dim; ++s) {
      const float b = tanhf(bcdt[s]);
      const float cc = tanhf(bcdt[state_dim + s]);
      const float half_dt = half_dt_min + sigmoidf_(bcdt[2 * state_dim + s]) * half_dt_range;
      const int hs = h * state_dim + s;
      const float mag = expf(2.0f * half_dt * decay[hs]);
      const float ang = 2.0f * half_dt * theta[hs];
      const float ar = mag * cosf(ang), ai = mag * sinf(ang);
      const size_t idx = (size_t)hs * head_dim + d;
      const float prev = prev_force[idx];
      const float sr = ssm_state[2 * idx], si = ssm_state[2 * idx + 1];
      const float force = b * value;
      const float dr = (force + ar * prev) * half_dt;
      const float di = (ai * prev) * half_dt;
      const float nr = sr * ar - si * ai + dr;
      const float ni = sr * ai + si * ar + di;
      ssm_state[2 * idx] = nr;
      ssm_state[2 * idx + 1] = ni;
      prev_force[idx] = force;
      total += cc * nr;
    }
    y[c] = (total + skip[c] * value) * sigmoidf_(mixer_in[hidden + c]);
  }
}

/* Latent attention step with the reference's decompressed fp32 cache (cpu_decoder.py:186-231):
 * mixer_in = [q (hidden) | latent | k_rope (heads*rope)], kv = [k_nope (heads*nope) | v (hidden)] (the
 * up-projection of the quantised latent), rope = [max_len][rope/2][2]. Appends k, v at `position`
 * and writes the attention output y [hidden]. */
static inline float round_half(float f) {
  /* fp32 -> fp16 (round to nearest even) -> fp32, for the reference GPU's fp16 K/V cache */
  uint32_t b;
  memcpy(&b, &f, 4);
  const uint32_t sign = b & 0x80000000u;
  const float a = fabsf(f);
  if (!(a < 65520.0f)) {
    float r = a != a ? a : INFINITY;
    uint32_t rb;
    memcpy(&rb, &r, 4);
    rb |= sign;
    memcpy(&r, &rb, 4);
    return r;
  }
  float r;
  if (a < 6.103515625e-05f) { /* subnormal half: quantum 2^-24 */
    r = rintf(a * 16777216.0f) / 16777216.0f;
  } else {
    int e;
    frexpf(a, &e);                     /* a in [2^(e-1), 2^e) */
    const float q = ldexpf(1.0f, e - 11); /* 10 fraction bits */
    r = rintf(a / q) * q;
  }
  uint32_t rb;
  memcpy(&rb, &r, 4);
  rb |= sign;
  memcpy(&r, &rb, 4);
  return r;
}

int orc_kv_half = 0; /* 1: store K and V rounded to fp16 as the reference GPU kernel does */

void orc_set_kv_half(int on) { orc_kv_half = on; }

void orc_attention_step(const float* mixer_in, const float* kv, const float* rope, int position, float* k_cache,
                        float* v_cache, int max_len, int heads, int head_dim, int nope, int rope_dim, int latent,
                        float scale, float* y) {
  const int hidden = heads * head_dim;
  float* q = (float*)malloc(sizeof(float) * (size_t)head_dim);
  float* key = (float*)malloc(sizeof(float) * (size_t)head_dim);
  float* scores = (float*)malloc(sizeof(float) * (size_t)(position + 1));
  for (int h = 0; h < heads; ++h) {
    for (int d = 0; d < nope; ++d) key[d] = kv[h * nope + d];
    for (int d = 0; d < rope_dim; ++d) key[nope + d] = mixer_in[hidden + latent + h * rope_dim + d];
    float* kc = k_cache + ((size_t)h * max_len) * head_dim;
    float* vc = v_cache + ((size_t)h * max_len) * head_dim;
    /* rotation: identity on the nope pairs, the rope table on the rope pairs */
    for (int pair = 0; pair < head_dim / 2; ++pair) {
      float cs = 1.0f, sn = 0.0f;
      if (2 * pair >= nope) {
        const int jr = pair - nope / 2;
        cs = rope[((size_t)position * (rope_dim / 2) + jr) * 2];
        sn = rope[((size_t)position * (rope_dim / 2) + jr) * 2 + 1];
      }
      const float q0 = mixer_in[h * head_dim + 2 * pair], q1 = mixer_in[h * head_dim + 2 * pair + 1];
      q[2 * pair] = (q0 * cs - q1 * sn) * scale;
      q[2 * pair + 1] = (q0 * sn + q1 * cs) * scale;
      const float k0 = key[2 * pair], k1 = key[2 * pair + 1];
      kc[(size_t)position * head_dim + 2 * pair] = k0 * cs - k1 * sn;
      kc[(size_t)position * head_dim + 2 * pair + 1] = k0 * sn + k1 * cs;
    }
    for (int d = 0; d < head_dim; ++d) vc[(size_t)position * head_dim + d] = kv[heads * nope + h * head_dim + d];
    if (orc_kv_half) {
      for (int d = 0; d < head_dim; ++d) {
        kc[(size_t)position * head_dim + d] = round_half(kc[(size_t)position * head_dim + d]);
        vc[(size_t)position * head_dim + d] = round_half(vc[(size_t)position * head_dim + d]);
      }
    }
    float peak = -INFINITY;
    for (int t = 0; t <= position; ++t) {
      float s = 0.0f;
      for (int d = 0; d < head_dim; ++d) s += q[d] * kc[(size_t)t * head_dim + d];
      scores[t] = s;
      if (s > peak) peak = s;
    }
    float norm = 0.0f;
    for (int t = 0; t <= position; ++t) {
      scores[t] = expf(scores[t] - peak);
      norm += scores[t];
    }
    for (int d = 0; d < head_dim; ++d) y[h * head_dim + d] = 0.0f;
    for (int t = 0; t <= position; ++t) {
      const float w = scores[t] / norm;
      for (int d = 0; d < head_dim; ++d) y[h * head_dim + d] += w * vc[(size_t)t * head_dim + d];
    }
  }
  free(q);
  free(key);
  free(scores);
}

/* ---- sampler -------------------------------------------------------------------------------- */

static void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
  /* Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3" (SC'11). */
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

/* Raw Philox4x32-10 block: out = philox(ctr[4], key[2]) (for known-answer tests). */
void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
  uint32_t c[4] = {ctr[0], ctr[1], ctr[2], ctr[3]};
  philox4x32_10(c, key[0], key[1]);
  memcpy(out, c, sizeof(c));
}

float orc_philox_uniform(uint64_t key, uint64_t counter) {
  uint32_t c[4] = {(uint32_t)counter, (uint32_t)(counter >> 32), 0x49766f6eu, 0u};
  philox4x32_10(c, (uint32_t)key, (uint32_t)(key >> 32));
  return (float)(c[0] >> 8) * (1.0f / 16777216.0f);
}

static inline uint32_t order_key(float v) {
  uint32_t b;
  memcpy(&b, &v, 4);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

/* e^x (x <= 0) for the sampler's candidate weights, the same operations as the kernels' sample_exp
 * (csrc/ivb_device.cuh), so the oracle weighs candidates bit for bit as the GPU does: Cody-Waite
 * reduction x = n ln2 + r with ln2 split into a 12-bit head (n * head exact) and a tail, e^r by the
 * degree-7 Taylor polynomial in Horner form with fmaf (|r| <= ln2/2), 2^n from the exponent field;
 * inputs below -87 give 0. */
static float sample_exp(float x) {
  if (!(x >= -87.0f)) return 0.0f;
  const float n = rintf(x * 0x1.715476p+0f);
  const float r = fmaf(-n, 0x1.0bfbe8p-15f, fmaf(-n, 0x1.62ep-1f, x));
  float p = 0x1.a01a02p-13f;
  p = fmaf(p, r, 0x1.6c16c2p-10f);
  p = fmaf(p, r, 0x1.111112p-7f);
  p = fmaf(p, r, 0x1.555556p-5f);
  p = fmaf(p, r, 0x1.555556p-3f);
  p = fmaf(p, r, 0x1p-1f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const uint32_t bits = (uint32_t)((int)n + 127) << 23;
  float scale;
  memcpy(&scale, &bits, 4);
  return p * scale;
}

typedef struct {
  uint32_t key;
  int32_t idx;
} Cand;

static int cand_cmp(const void* a, const void* b) {
  const Cand* x = (const Cand*)a;
  const Cand* y = (const Cand*)b;
  if (x->key != y->key) return x->key > y->key ? -1 : 1;
  return x->idx < y->idx ? -1 : (x->idx > y->idx ? 1 : 0);
}

/* score = logit * (1/T); seen: score *= score > 0 ? ipen : pen (reference ternary.cu:989-995).
 * The K = clamp(top_k, 1, min(max_top_k, vocab, 1024)) best by (score desc, index asc);
 * p_c = sample_exp(s_c - s_0); cdf in 32-candidate chunks (Hillis-Steele inclusive scan inside a chunk,
 * chunk totals carried in order); u = philox(rng[0], rng[1]) (counter then incremented),
 * target = min(u, 0.99999994) * cdf[K-1], token = #(cdf <= target) clamped to K - 1.
 * Sets seen[token] = 1 and returns the token. */
int64_t orc_sample(const float* logits, uint8_t* seen, int vocab, float temperature, float penalty,
                   float inverse_penalty, int64_t top_k, int max_top_k, uint64_t* rng) {
  const float inv_t = 1.0f / temperature;
  Cand* all = (Cand*)malloc(sizeof(Cand) * (size_t)vocab);
  for (int i = 0; i < vocab; ++i) {
    float s = logits[i] * inv_t;
    if (seen[i]) s *= s > 0.0f ? inverse_penalty : penalty;
    all[i].key = order_key(s);
    all[i].idx = i;
  }
  int cap = max_top_k < vocab ? max_top_k : vocab;
  if (cap > 1024) cap = 1024;
  const int K = (int)(top_k < 1 ? 1 : (top_k > cap ? cap : top_k));
  qsort(all, (size_t)vocab, sizeof(Cand), cand_cmp);
  float* cdf = (float*)malloc(sizeof(float) * (size_t)K);
  float top;
  {
    uint32_t k = all[0].key;
    uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    memcpy(&top, &b, 4);
  }
  for (int c = 0; c < K; ++c) {
    const uint32_t k = all[c].key;
    const uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    float s;
    memcpy(&s, &b, 4);
    cdf[c] = sample_exp(s - top);
  }
  float carry = 0.0f;
  for (int base = 0; base < K; base += 32) {
    float v[32], nv[32];
    for (int l = 0; l < 32; ++l) v[l] = base + l < K ? cdf[base + l] : 0.0f;
    for (int off = 1; off < 32; off <<= 1) {
      for (int l = 0; l < 32; ++l) nv[l] = l >= off ? v[l] + v[l - off] : v[l];
      memcpy(v, nv, sizeof(v));
    }
    for (int l = 0; l < 32 && base + l < K; ++l) cdf[base + l] = carry + v[l];
    carry = carry + v[31];
  }
  float u = orc_philox_uniform(rng[0], rng[1]);
  rng[1] += 1;
  if (u > 0.99999994f) u = 0.99999994f;
  const float target = u * cdf[K - 1];
  int below = 0;
  for (int c = 0; c < K; ++c) below += cdf[c] <= target ? 1 : 0;
  const int chosen = below < K - 1 ? below : K - 1;
  const int64_t token = all[chosen].idx;
  seen[token] = 1;
  free(cdf);
  free(all);
  return token;
}

int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
