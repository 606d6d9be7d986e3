/*
 * TEST INFRASTRUCTURE ONLY -- the CPU checker for the NVFP4 QSA CUDA path.
 *
 * A plain-C restatement of the reference's algorithms for this path:
 *   - the NVFP4 codec oracle      python/nvfp4_qsa/oracle.py (== src/nvfp4_oracle.py)
 *   - the paged writer's contract python/nvfp4_qsa/kernels.py:46-165
 *   - the sparse reader's contract python/nvfp4_qsa/kernels.py:168-403,
 *     computed in float64 like the reference's FP32/64 QSA reference
 *     src/qsa_ref.py:12-52
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load
 * this file's library, and only as the checker / the timed CPU baseline.
 * The product (nvfp4-qsa_b200/) never links or imports it.
 *
 * Parity pin: tests/golden/ holds vectors produced by the reference's own
 * Python oracle and qsa_reference (tests/golden/make_golden.py); the CPU test
 * suite checks this restatement against them byte for byte (codec) and to
 * 1e-5 (attention).
 *
 * Build: oracle/build.py (gcc -O2 -fopenmp -ffp-contract=off, no fast-math).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define E2M1_MAX 6.0f  /* oracle.py:20 */
#define E4M3_MAX 448.0f /* oracle.py:21 */

static const float kGrid[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f}; /* oracle.py:19 */

static inline float f32_from_bits(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static inline uint32_t bits_from_f32(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static inline float bf16_to_f32(uint16_t b) { return f32_from_bits((uint32_t)b << 16); }

/* fp32 -> float8_e4m3fn byte, round-to-nearest-even, as torch's
 * Tensor.to(torch.float8_e4m3fn) does for the clamped block scales of
 * oracle.py:55 (inputs are NaN or in [-448, 448] there). */
uint8_t orc_f32_to_e4m3(float x) {
  const uint32_t u = bits_from_f32(x);
  const uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
  float a = fabsf(x);
  if (a != a) return (uint8_t)(0x7f | sign);
  if (a > E4M3_MAX) a = E4M3_MAX;
  if (a < 0.015625f) { /* subnormal range: multiples of 2^-9 */
    const float q = rintf(a * 512.0f);
    return (uint8_t)(sign | (uint8_t)q); /* q == 8 encodes 2^-6 exactly */
  }
  int e;
  const float m = frexpf(a, &e); /* a = m * 2^e, m in [0.5, 1) */
  (void)m;
  e -= 1;                                 /* a = f * 2^e, f in [1, 2) */
  float r = rintf(ldexpf(a, 3 - e));      /* in [8, 16] */
  if (r >= 16.0f) {
    r = 8.0f;
    e += 1;
  }
  uint32_t code = ((uint32_t)(e + 7) << 3) | ((uint32_t)r - 8u);
  if (code > 0x7e) code = 0x7e;
  return (uint8_t)(sign | code);
}

/* float8_e4m3fn byte -> fp32 (exact). */
float orc_e4m3_to_f32(uint8_t b) {
  const int sign = b >> 7, exp = (b >> 3) & 0xf, man = b & 7;
  float v;
  if (exp == 0xf && man == 7) return f32_from_bits(sign ? 0xffc00000u : 0x7fc00000u);
  if (exp == 0)
    v = ldexpf((float)man, -9);
  else
    v = ldexpf(8.0f + (float)man, exp - 10);
  return sign ? -v : v;
}

/* _round_e2m1_magnitude (oracle.py:30-44) + sign (oracle.py:62) for a value
 * already clamped to [-6, 6] (NaN passes through and yields code 0). */
uint8_t orc_e2m1_code(float y) {
  const float a = fabsf(y);
  uint8_t m = 0;
  if (a > 0.25f && a < 0.75f) m = 1;
  if (a >= 0.75f && a <= 1.25f) m = 2;
  if (a > 1.25f && a < 1.75f) m = 3;
  if (a >= 1.75f && a <= 2.5f) m = 4;
  if (a > 2.5f && a < 3.5f) m = 5;
  if (a >= 3.5f && a <= 5.0f) m = 6;
  if (a > 5.0f) m = 7;
  return (uint8_t)(((y < 0.0f) ? 8 : 0) | m);
}

/* One group of `block` values -> scale byte + `block` codes (oracle.py:51-63). */
static uint8_t encode_group(const float* x, int block, float g, uint8_t* codes, int64_t* clip, int64_t* sat) {
  float amax = 0.0f; /* xg.abs().amax(): NaN propagates */
  int has_nan = 0;
  for (int i = 0; i < block; ++i) {
    const float a = fabsf(x[i]);
    if (a != a) has_nan = 1;
    if (a > amax) amax = a;
  }
  if (has_nan) amax = f32_from_bits(0x7fc00000u);
  float bs = g * amax;
  bs = bs / E2M1_MAX; /* oracle.py:54: g * group_amax / E2M1_MAX */
  if (bs > E4M3_MAX) bs = E4M3_MAX;
  if (bs < -E4M3_MAX) bs = -E4M3_MAX;
  if (sat && fabsf(bs) >= 447.999f) ++*sat; /* oracle.py:64 */
  const uint8_t byte = orc_f32_to_e4m3(bs);
  const float bs_f32 = orc_e4m3_to_f32(byte);
  const float den = (bs_f32 < 1e-30f) ? 1e-30f : bs_f32; /* clamp_min(1e-30), NaN stays */
  const float out_scale = g / den;                        /* oracle.py:57 */
  for (int i = 0; i < block; ++i) {
    float y = x[i] * out_scale;
    if (clip && fabsf(y) > E2M1_MAX) ++*clip; /* oracle.py:59 */
    if (y > E2M1_MAX) y = E2M1_MAX;
    if (y < -E2M1_MAX) y = -E2M1_MAX;
    codes[i] = orc_e2m1_code(y);
  }
  return byte;
}

/* encode (oracle.py:47-69): x fp32 [m, n] contiguous. */
void orc_encode_rows(const float* x, int64_t m, int64_t n, int32_t block, float g, uint8_t* nibbles,
                     uint8_t* packed, uint8_t* scales, int64_t* counts) {
  const int64_t groups = m * (n / block);
  int64_t clip = 0, sat = 0;
  uint8_t codes[4096];
  for (int64_t gi = 0; gi < groups; ++gi) {
    const float* xp = x + gi * block;
    scales[gi] = encode_group(xp, block, g, codes, &clip, &sat);
    for (int i = 0; i < block; i += 2) {
      const int64_t e = gi * block + i;
      packed[e >> 1] = (uint8_t)(codes[i] | (codes[i + 1] << 4)); /* oracle.py:65-66 */
      if (nibbles) {
        nibbles[e] = codes[i];
        nibbles[e + 1] = codes[i + 1];
      }
    }
  }
  if (counts) {
    counts[0] += clip;
    counts[1] += sat;
  }
}

/* decode (oracle.py:72-85): fp4 * (bs / g). */
void orc_decode_rows(const uint8_t* packed, const uint8_t* scales, int64_t m, int64_t n, int32_t block, float g,
                     float* out) {
  for (int64_t e = 0; e < m * n; ++e) {
    const uint8_t byte = packed[e >> 1];
    const uint8_t nib = (e & 1) ? (byte >> 4) : (byte & 0xf);
    const float sign = (nib & 8) ? -1.0f : 1.0f;
    const float fp4 = kGrid[nib & 7] * sign;
    const float f = orc_e4m3_to_f32(scales[e / block]) / g;
    out[e] = fp4 * f;
  }
}

/* Paged writer contract (kernels.py:46-165) with the oracle's encoding.
 * key/value: bf16 bits [tokens, kv_heads, head_dim] with element strides. */
void orc_write_cache(const uint16_t* key, int64_t key_st, int64_t key_sh, const uint16_t* value, int64_t val_st,
                     int64_t val_sh, uint8_t* kd, int64_t kd_sb, int64_t kd_st, int64_t kd_sh, uint8_t* ks,
                     int64_t ks_sb, int64_t ks_st, int64_t ks_sh, uint8_t* vd, int64_t vd_sb, int64_t vd_st,
                     int64_t vd_sh, uint8_t* vs, int64_t vs_sb, int64_t vs_st, int64_t vs_sh, const int64_t* slots,
                     int64_t tokens, int32_t kv_heads, int32_t head_dim, int64_t num_blocks, int64_t page_size,
                     float gk, float gv) {
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < tokens; ++t) {
    const int64_t slot = slots[t];
    if (slot < 0) continue; /* kernels.py:71-77 */
    const int64_t blk = slot / page_size, off = slot % page_size;
    if (blk >= num_blocks) continue;
    float x[4096];
    uint8_t codes[4096];
    for (int h = 0; h < kv_heads; ++h) {
      for (int r = 0; r < 2; ++r) {
        const uint16_t* src = r ? value + t * val_st + h * val_sh : key + t * key_st + h * key_sh;
        uint8_t* drow = r ? vd + blk * vd_sb + off * vd_st + h * vd_sh : kd + blk * kd_sb + off * kd_st + h * kd_sh;
        uint8_t* srow = r ? vs + blk * vs_sb + off * vs_st + h * vs_sh : ks + blk * ks_sb + off * ks_st + h * ks_sh;
        const float g = r ? gv : gk;
        for (int d = 0; d < head_dim; ++d) x[d] = bf16_to_f32(src[d]);
        for (int grp = 0; grp < head_dim / 16; ++grp) {
          srow[grp] = encode_group(x + 16 * grp, 16, g, codes + 16 * grp, NULL, NULL);
        }
        for (int j = 0; j < head_dim / 2; ++j) drow[j] = (uint8_t)(codes[2 * j] | (codes[2 * j + 1] << 4));
      }
    }
  }
}

/* bf16 round-to-nearest-even of an fp32 value (NaN -> 0x7fff, the sm_100a
 * conversion's canonical NaN). */
static inline uint16_t bf16_rn_bits(float f) {
  const uint32_t u = bits_from_f32(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fff;
  return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}
static inline float bf16_round(float f) { return bf16_to_f32(bf16_rn_bits(f)); }

/* K-norm + rotary embedding ahead of the writer: the K path of the
 * reference's caller (integration/snapshot/qsa.py:618-667), vLLM's
 * GemmaRMSNorm (ir rms_norm: fp32, x * rsqrt(mean(x^2) + eps) * (w + 1), to
 * bf16) and native rotary embedding (bf16 tensor arithmetic: every product
 * and sum rounded to bf16), with the summation order and the square root /
 * divide that nvqsa_norm_rope_write_cache specifies: 32 partial sums, partial
 * l over elements [l*E, l*E+E) (E = head_dim/32) as (fmaf-sum of the squares
 * of its even elements, in order) + (the same over its odd elements), then
 * added pairwise at distances 16, 8, 4, 2, 1; r = 1 / sqrtf(ss / head_dim + eps).
 * key: bf16 bits with element strides; out: bf16 bits [tokens, kv_heads,
 * head_dim] contiguous; valid[t] = 0 for a position outside [0, max_pos)
 * (the token is skipped: its out rows are left as they are). */
void orc_norm_rope(const uint16_t* key, int64_t st, int64_t sh, int64_t tokens, int32_t kv_heads, int32_t head_dim,
                   const float* weight, float offset, float eps, const int64_t* positions, const uint16_t* cos_sin,
                   int64_t cs_stride, int64_t max_pos, int32_t rot, int32_t neox, uint16_t* out, uint8_t* valid) {
  const int E = head_dim / 32;
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < tokens; ++t) {
    int64_t pos = 0;
    if (rot > 0) {
      pos = positions[t];
      if (pos < 0 || pos >= max_pos) {
        valid[t] = 0;
        continue;
      }
    }
    valid[t] = 1;
    for (int h = 0; h < kv_heads; ++h) {
      const uint16_t* src = key + t * st + h * sh;
      float y[4096];
      for (int d = 0; d < head_dim; ++d) y[d] = bf16_to_f32(src[d]);
      if (weight) {
        float part[32];
        for (int l = 0; l < 32; ++l) {
          float even = 0.0f, odd = 0.0f;
          for (int j = 0; j < E; j += 2) {
            even = fmaf(y[l * E + j], y[l * E + j], even);
            odd = fmaf(y[l * E + j + 1], y[l * E + j + 1], odd);
          }
          part[l] = even + odd;
        }
        for (int m = 16; m >= 1; m >>= 1)
          for (int l = 0; l < m; ++l) part[l] = part[l] + part[l + m];
        const float r = 1.0f / sqrtf(part[0] * (1.0f / (float)head_dim) + eps);
        for (int d = 0; d < head_dim; ++d) y[d] = bf16_round((y[d] * r) * (weight[d] + offset));
      }
      if (rot > 0) {
        const uint16_t* cs = cos_sin + pos * cs_stride;
        const int half = rot / 2;
        float o[4096];
        memcpy(o, y, sizeof(float) * (size_t)head_dim);
        for (int i = 0; i < half; ++i) {
          const int i1 = neox ? i : 2 * i, i2 = neox ? i + half : 2 * i + 1;
          const float c = bf16_to_f32(cs[i]), s = bf16_to_f32(cs[half + i]);
          const float x1 = y[i1], x2 = y[i2];
          o[i1] = bf16_round(bf16_round(x1 * c) - bf16_round(x2 * s));
          o[i2] = bf16_round(bf16_round(x2 * c) + bf16_round(x1 * s));
        }
        memcpy(y, o, sizeof(float) * (size_t)head_dim);
      }
      uint16_t* dst = out + (t * kv_heads + h) * head_dim;
      for (int d = 0; d < head_dim; ++d) dst[d] = bf16_rn_bits(y[d]);
    }
  }
}

/* Sparse paged GQA decode attention (kernels.py:168-345 masking; math in
 * float64 as src/qsa_ref.py:12-52).  out: fp32 [rows, query_heads, head_dim]
 * contiguous; lse_out (optional, fp32 [rows, query_heads]) receives each
 * head's base-2 log-sum-exp, or -inf when no selection is valid.  K/V are dequantised exactly (e2m1 * e4m3); the score scale is
 * head_dim^-0.5 / gk and the output is divided by gv. */
static void attention_core(int fp8, const uint16_t* q, int64_t q_sr, int64_t q_sh, const uint8_t* kd, int64_t kd_sb,
                          int64_t kd_st, int64_t kd_sh, const uint8_t* ks, int64_t ks_sb, int64_t ks_st,
                          int64_t ks_sh, const uint8_t* vd, int64_t vd_sb, int64_t vd_st, int64_t vd_sh,
                          const uint8_t* vs, int64_t vs_sb, int64_t vs_st, int64_t vs_sh, int64_t num_blocks,
                          int64_t page_size, int32_t kv_heads, double score_mul, double out_mul, const int32_t* indices,
                          int64_t topk, const int32_t* block_table, int64_t num_requests, int64_t table_width,
                          const int32_t* token_to_request, float* out, int64_t rows, int32_t query_heads,
                          int32_t head_dim, float* lse_out) {
  const int G = query_heads / kv_heads;
  const double scale = score_mul / sqrt((double)head_dim);
#pragma omp parallel for collapse(2) schedule(dynamic)
  for (int64_t r = 0; r < rows; ++r) {
    for (int h = 0; h < kv_heads; ++h) {
      const int32_t req = token_to_request[r];
      const int req_ok = req >= 0 && (int64_t)req < num_requests;
      int64_t* sel_blk = (int64_t*)malloc(sizeof(int64_t) * (topk > 0 ? topk : 1));
      int64_t* sel_off = (int64_t*)malloc(sizeof(int64_t) * (topk > 0 ? topk : 1));
      int64_t nv = 0;
      for (int64_t i = 0; i < topk && req_ok; ++i) { /* kernels.py:236-257 */
        const int32_t idx = indices[r * topk + i];
        if (idx < 0) continue;
        const int64_t lpage = (int64_t)idx / page_size;
        if (lpage >= table_width) continue;
        const int32_t phys = block_table[(int64_t)req * table_width + lpage];
        if (phys < 0 || (int64_t)phys >= num_blocks) continue;
        sel_blk[nv] = phys;
        sel_off[nv] = (int64_t)idx - lpage * page_size;
        ++nv;
      }
      double* K = (double*)malloc(sizeof(double) * (nv > 0 ? nv : 1) * head_dim);
      double* V = (double*)malloc(sizeof(double) * (nv > 0 ? nv : 1) * head_dim);
      double* s = (double*)malloc(sizeof(double) * (nv > 0 ? nv : 1));
      for (int64_t t = 0; t < nv; ++t) {
        const int64_t b = sel_blk[t], o = sel_off[t];
        const uint8_t* kdr = kd + b * kd_sb + o * kd_st + h * kd_sh;
        const uint8_t* ksr = ks + b * ks_sb + o * ks_st + h * ks_sh;
        const uint8_t* vdr = vd + b * vd_sb + o * vd_st + h * vd_sh;
        const uint8_t* vsr = vs + b * vs_sb + o * vs_st + h * vs_sh;
        for (int d = 0; d < head_dim; ++d) {
          if (fp8 == 2) { /* bf16 element (the BF16 sibling reader, integration/snapshot/qsa.py:352-366) */
            uint16_t kb2, vb2;
            memcpy(&kb2, kdr + 2 * d, 2);
            memcpy(&vb2, vdr + 2 * d, 2);
            K[t * head_dim + d] = (double)bf16_to_f32(kb2);
            V[t * head_dim + d] = (double)bf16_to_f32(vb2);
            continue;
          }
          if (fp8) { /* one float8_e4m3fn byte per element (qsa_fp8_harness.py:139-158) */
            K[t * head_dim + d] = (double)orc_e4m3_to_f32(kdr[d]);
            V[t * head_dim + d] = (double)orc_e4m3_to_f32(vdr[d]);
            continue;
          }
          const uint8_t kb = kdr[d >> 1], vb = vdr[d >> 1];
          const uint8_t kn = (d & 1) ? (kb >> 4) : (kb & 0xf);
          const uint8_t vn = (d & 1) ? (vb >> 4) : (vb & 0xf);
          const double kv = (kn & 8 ? -1.0 : 1.0) * kGrid[kn & 7] * (double)orc_e4m3_to_f32(ksr[d >> 4]);
          const double vv = (vn & 8 ? -1.0 : 1.0) * kGrid[vn & 7] * (double)orc_e4m3_to_f32(vsr[d >> 4]);
          K[t * head_dim + d] = kv;
          V[t * head_dim + d] = vv;
        }
      }
      for (int j = 0; j < G; ++j) {
        const int qh = h * G + j;
        const uint16_t* qr = q + r * q_sr + qh * q_sh;
        float* orow = out + (r * query_heads + qh) * head_dim;
        if (nv == 0) { /* kernels.py:333-337: no valid selection -> zeros */
          for (int d = 0; d < head_dim; ++d) orow[d] = 0.0f;
          if (lse_out) lse_out[r * query_heads + qh] = -INFINITY;
          continue;
        }
        double mx = -INFINITY;
        for (int64_t t = 0; t < nv; ++t) {
          double acc = 0.0;
          for (int d = 0; d < head_dim; ++d) acc += (double)bf16_to_f32(qr[d]) * K[t * head_dim + d];
          s[t] = acc * scale;
          if (s[t] > mx) mx = s[t];
        }
        double den = 0.0;
        for (int64_t t = 0; t < nv; ++t) {
          s[t] = exp(s[t] - mx);
          den += s[t];
        }
        for (int d = 0; d < head_dim; ++d) {
          double acc = 0.0;
          for (int64_t t = 0; t < nv; ++t) acc += s[t] * V[t * head_dim + d];
          orow[d] = (float)(acc / den * out_mul);
        }
        /* base-2 log-sum-exp of the scaled scores, the split-KV partial format of
         * src/qsa_fp8_harness.py:183-208 (lse = m + log2 l in log2 units) */
        if (lse_out) lse_out[r * query_heads + qh] = (float)(mx / log(2.0) + log2(den));
      }
      free(sel_blk);
      free(sel_off);
      free(K);
      free(V);
      free(s);
    }
  }
}

void orc_sparse_attention(const uint16_t* q, int64_t q_sr, int64_t q_sh, const uint8_t* kd, int64_t kd_sb,
                          int64_t kd_st, int64_t kd_sh, const uint8_t* ks, int64_t ks_sb, int64_t ks_st,
                          int64_t ks_sh, const uint8_t* vd, int64_t vd_sb, int64_t vd_st, int64_t vd_sh,
                          const uint8_t* vs, int64_t vs_sb, int64_t vs_st, int64_t vs_sh, int64_t num_blocks,
                          int64_t page_size, int32_t kv_heads, float gk, float gv, const int32_t* indices,
                          int64_t topk, const int32_t* block_table, int64_t num_requests, int64_t table_width,
                          const int32_t* token_to_request, float* out, int64_t rows, int32_t query_heads,
                          int32_t head_dim, float* lse_out) {
  attention_core(0, q, q_sr, q_sh, kd, kd_sb, kd_st, kd_sh, ks, ks_sb, ks_st, ks_sh, vd, vd_sb, vd_st, vd_sh, vs,
                 vs_sb, vs_st, vs_sh, num_blocks, page_size, kv_heads, 1.0 / (double)gk, 1.0 / (double)gv, indices,
                 topk, block_table, num_requests, table_width, token_to_request, out, rows, query_heads, head_dim,
                 lse_out);
}

/* The FP8 sibling reader (src/qsa_fp8_harness.py:42-208): K and V caches of
 * float8_e4m3fn bytes [blocks, page, kv_heads, head_dim] with byte strides;
 * the per-tensor k_scale multiplies the scores (folded into the softmax scale,
 * :101-102), v_scale the normalised output (:175).  Same masking, softmax and
 * partial format as the NVFP4 reader. */
void orc_sparse_attention_fp8(const uint16_t* q, int64_t q_sr, int64_t q_sh, const uint8_t* kc, int64_t kc_sb,
                              int64_t kc_st, int64_t kc_sh, const uint8_t* vc, int64_t vc_sb, int64_t vc_st,
                              int64_t vc_sh, int64_t num_blocks, int64_t page_size, int32_t kv_heads, float k_scale,
                              float v_scale, const int32_t* indices, int64_t topk, const int32_t* block_table,
                              int64_t num_requests, int64_t table_width, const int32_t* token_to_request,
                              float* out, int64_t rows, int32_t query_heads, int32_t head_dim, float* lse_out) {
  attention_core(1, q, q_sr, q_sh, kc, kc_sb, kc_st, kc_sh, kc, kc_sb, kc_st, kc_sh, vc, vc_sb, vc_st, vc_sh, vc,
                 vc_sb, vc_st, vc_sh, num_blocks, page_size, kv_heads, (double)k_scale, (double)v_scale, indices,
                 topk, block_table, num_requests, table_width, token_to_request, out, rows, query_heads, head_dim,
                 lse_out);
}

/* The BF16 sibling reader: bf16 K and V caches [blocks, page, kv_heads, head_dim]
 * with byte strides; plain scale head_dim^-0.5 (src/qsa_ref.py:12-52 on a bf16
 * cache).  Same masking, softmax and partial format as the NVFP4 reader. */
void orc_sparse_attention_bf16(const uint16_t* q, int64_t q_sr, int64_t q_sh, const uint8_t* kc, int64_t kc_sb,
                               int64_t kc_st, int64_t kc_sh, const uint8_t* vc, int64_t vc_sb, int64_t vc_st,
                               int64_t vc_sh, int64_t num_blocks, int64_t page_size, int32_t kv_heads,
                               const int32_t* indices, int64_t topk, const int32_t* block_table,
                               int64_t num_requests, int64_t table_width, const int32_t* token_to_request,
                               float* out, int64_t rows, int32_t query_heads, int32_t head_dim, float* lse_out) {
  attention_core(2, q, q_sr, q_sh, kc, kc_sb, kc_st, kc_sh, kc, kc_sb, kc_st, kc_sh, vc, vc_sb, vc_st, vc_sh, vc,
                 vc_sb, vc_st, vc_sh, num_blocks, page_size, kv_heads, 1.0, 1.0, indices, topk, block_table,
                 num_requests, table_width, token_to_request, out, rows, query_heads, head_dim, lse_out);
}

void orc_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int orc_get_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
