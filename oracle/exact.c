/*
 * oracle/exact.c — TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * Scalar CPU restatement of the reference's sparse-selection algorithm in the
 * exact arithmetic order the CUDA kernels use, so that GPU results can be
 * compared bit for bit.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg load this library.  Build: oracle/Makefile (no fp
 * contraction: -ffp-contract=off, SSE float arithmetic).
 *
 * Each function cites the reference code it restates (paths inside the
 * reference project; hi/ = source/headinfer/headinfer/).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---- 16-bit float conversions (round to nearest even) ---------------------- */

static float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do {
        ++e;
        man <<= 1;
      } while ((man & 0x400u) == 0);
      man &= 0x3ffu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 0x1f) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp - 15 + 127) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static uint16_t f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t a = x & 0x7fffffffu;
  if (a >= 0x7f800000u) return (uint16_t)(sign | (a > 0x7f800000u ? 0x7e00u : 0x7c00u));
  if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 -> inf */
  if (a < 0x38800000u) {                                    /* below 2^-14: subnormal */
    if (a < 0x33000000u) return (uint16_t)sign;             /* <= 2^-25 -> 0 (2^-25 ties to even) */
    uint32_t e = a >> 23;
    uint32_t m = (a & 0x7fffffu) | 0x800000u;
    int shift = 126 - (int)e;
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
  }
  uint32_t e = (a >> 23) - 127 + 15;
  uint32_t m = a & 0x7fffffu;
  uint32_t q = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;
  return (uint16_t)(sign | q);
}

static float bf16_to_f32(uint16_t h) {
  uint32_t bits = (uint32_t)h << 16;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static uint16_t f32_to_bf16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
  x += 0x7fffu + ((x >> 16) & 1u);
  return (uint16_t)(x >> 16);
}

/* dtype: 0 = fp16, 1 = bf16 (stored as uint16) */
static float to_f32(uint16_t v, int dtype) { return dtype == 0 ? f16_to_f32(v) : bf16_to_f32(v); }
static uint16_t from_f32(float v, int dtype) { return dtype == 0 ? f32_to_f16(v) : f32_to_bf16(v); }

float orc_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
uint16_t orc_f32_to_f16(float f) { return f32_to_f16(f); }
uint16_t orc_f32_to_bf16(float f) { return f32_to_bf16(f); }

/* ---- Quest page metadata --------------------------------------------------------
 * hi/quest_offload_cache.py:276-289: tail = K[sink:]; complete pages of
 * block rows; page_min/max = amin/amax over the page per channel.
 * keys: [n_tokens][D]; writes n_pages = (n_tokens - sink) / block pages. */
int orc_quest_page_metadata(const uint16_t* keys, int64_t n_tokens, int D, int sink, int block,
                            int dtype, uint16_t* pmin, uint16_t* pmax) {
  if (n_tokens <= sink) return 0;
  int64_t pages = (n_tokens - sink) / block;
  for (int64_t p = 0; p < pages; ++p) {
    for (int d = 0; d < D; ++d) {
      const uint16_t* col = keys + (sink + p * block) * (int64_t)D + d;
      uint16_t vmin = col[0], vmax = col[0];
      float fmin = to_f32(vmin, dtype), fmax = fmin;
      for (int t = 1; t < block; ++t) {
        uint16_t x = col[(int64_t)t * D];
        float fx = to_f32(x, dtype);
        if (fx < fmin) { fmin = fx; vmin = x; }
        if (fx > fmax) { fmax = fx; vmax = x; }
      }
      pmin[p * D + d] = vmin;
      pmax[p * D + d] = vmax;
    }
  }
  return (int)pages;
}

/* ---- INT4 affine quantiser ----------------------------------------------------------
 * hi/twilight_offload_cache.py:25-37 applied to K.view(-1, group):
 * mn/mx per group; scale = ((mx - mn) in K dtype).float().clamp_min(1e-9) / 15
 * -> K dtype; code = clamp(round((k - mn) / scale), 0, 15); byte j = code[2j] |
 * code[2j+1] << 4.  scale_div 0: "/ 15" as x * (1/15) (torch on CUDA with a
 * CPU-scalar divisor); 1: IEEE divide (torch on CPU). */
void orc_int4_pack(const uint16_t* keys, int64_t n_tokens, int D, int group, int dtype,
                   int scale_div, uint8_t* packed, uint16_t* scale, uint16_t* minimum) {
  const int ngroups = D / group;
  const float inv15 = 1.0f / 15.0f;
  for (int64_t t = 0; t < n_tokens; ++t) {
    const uint16_t* row = keys + t * D;
    for (int gi = 0; gi < ngroups; ++gi) {
      const uint16_t* gr = row + gi * group;
      float mn = to_f32(gr[0], dtype), mx = mn;
      for (int i = 1; i < group; ++i) {
        float x = to_f32(gr[i], dtype);
        mn = fminf(mn, x);
        mx = fmaxf(mx, x);
      }
      float diff = to_f32(from_f32(mx - mn, dtype), dtype);
      float clamped = fmaxf(diff, 1e-9f);
      float sc32 = scale_div ? clamped / 15.0f : clamped * inv15;
      uint16_t sc_t = from_f32(sc32, dtype);
      float sc = to_f32(sc_t, dtype);
      scale[t * ngroups + gi] = sc_t;
      minimum[t * ngroups + gi] = from_f32(mn, dtype);
      for (int i = 0; i < group; i += 2) {
        uint32_t c[2];
        for (int j = 0; j < 2; ++j) {
          float x = to_f32(gr[i + j], dtype);
          float v = rintf((x - mn) / sc);
          if (!(v >= 0.0f)) v = 0.0f;
          if (v > 15.0f) v = 15.0f;
          c[j] = (uint32_t)v;
        }
        packed[t * (D / 2) + (gi * group + i) / 2] = (uint8_t)(c[0] | (c[1] << 4));
      }
    }
  }
}

/* ---- Quest upper-bound score ----------------------------------------------------------
 * hi/twilight_fused_quest.py:13-32 (== the torch expression of
 * hi/twilight_offload_cache.py:1148-1149 on CUDA): per lane l (0..31) the
 * products at d = l, l+32, l+64, l+96 are added to 0 in that order; then lane
 * sums combine as v[l] += v[l + 2^s] for s = 0..4 (lane 0 result).
 * q: [G][R][D] fp32; pmin/pmax: [G][meta_group_stride] (page p at p*D). */
void orc_quest_score(const float* q, const uint16_t* pmin, const uint16_t* pmax, int G, int R,
                     int P, int64_t meta_group_stride, int dtype, float* scores) {
  const int D = 128;
  for (int g = 0; g < G; ++g) {
    for (int r = 0; r < R; ++r) {
      const float* qr = q + ((int64_t)g * R + r) * D;
      for (int p = 0; p < P; ++p) {
        const uint16_t* mn = pmin + g * meta_group_stride + (int64_t)p * D;
        const uint16_t* mx = pmax + g * meta_group_stride + (int64_t)p * D;
        float lane[32];
        for (int l = 0; l < 32; ++l) {
          float acc = 0.0f;
          for (int c = 0; c < 4; ++c) {
            int d = l + 32 * c;
            float e = qr[d] > 0.0f ? to_f32(mx[d], dtype) : to_f32(mn[d], dtype);
            float prod = e * qr[d];
            acc = acc + prod;
          }
          lane[l] = acc;
        }
        for (int off = 1; off < 32; off <<= 1) {
          float next[32];
          for (int l = 0; l < 32; ++l) next[l] = (l + off < 32) ? lane[l] + lane[l + off] : lane[l];
          memcpy(lane, next, sizeof(lane));
        }
        scores[((int64_t)g * R + r) * P + p] = lane[0];
      }
    }
  }
}

/* ---- top-k pages --------------------------------------------------------------------------
 * hi/twilight_offload_cache.py:1153-1155 (torch.topk sorted=False) and
 * hi/quest_offload_cache.py:373-374 (then sorted).  A set: the k largest scores,
 * ties at the k-th value resolved towards lower page ids; output ascending. */
typedef struct {
  uint32_t key;
  int32_t idx;
} keyed_t;

static uint32_t float_key(float f) {
  if (f == 0.0f) f = 0.0f;
  uint32_t u;
  memcpy(&u, &f, 4);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

static float key_float(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static int cmp_desc_key_asc_idx(const void* a, const void* b) {
  const keyed_t* x = (const keyed_t*)a;
  const keyed_t* y = (const keyed_t*)b;
  if (x->key != y->key) return x->key > y->key ? -1 : 1;
  return x->idx < y->idx ? -1 : (x->idx > y->idx);
}

static int cmp_i32(const void* a, const void* b) {
  int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
  return x < y ? -1 : (x > y);
}

void orc_topk_pages(const float* scores, int rows, int n, int k, int32_t* out) {
  keyed_t* buf = (keyed_t*)malloc(sizeof(keyed_t) * (size_t)(n > 0 ? n : 1));
  for (int r = 0; r < rows; ++r) {
    for (int i = 0; i < n; ++i) {
      buf[i].key = float_key(scores[(int64_t)r * n + i]);
      buf[i].idx = i;
    }
    qsort(buf, (size_t)n, sizeof(keyed_t), cmp_desc_key_asc_idx);
    int32_t* dst = out + (int64_t)r * k;
    for (int i = 0; i < k; ++i) dst[i] = buf[i].idx;
    qsort(dst, (size_t)k, sizeof(int32_t), cmp_i32);
  }
  free(buf);
}

/* ---- INT4 QK estimate ------------------------------------------------------------------------
 * hi/twilight_fused_qk.py:13-31 (dequant k = code*scale + min in fp32, no FMA)
 * and hi/twilight_offload_cache.py:1197-1263 (QK) + :1261 (/ sqrt(D), applied
 * as torch on CUDA does: x * (1 / (float)sqrt(D))).  The dot accumulates with
 * fused multiply-adds, as the fp32 GEMV of torch.matmul
 * (hi/twilight_offload_cache.py:1257) does on CUDA.  Reduction order: part j
 * (j = 0..3) covers channels 32j..32j+31; channel 32j + i goes to
 * accumulator i % 4 (acc = fma(k, q, acc), i in order from 0), and the part
 * is (acc0 + acc1) + (acc2 + acc3); then (s0 + s1) + (s2 + s3).  Candidate n of row (g, r) is token
 * sink + pages[g][r][n / block] * block + n % block of entry g. */
void orc_int4_qk(const float* q, const uint8_t* packed, const uint16_t* scale,
                 const uint16_t* minimum, int64_t entry_stride, const int32_t* pages, int G, int R,
                 int b0, int block, int sink, int group, int dtype, float* logits) {
  const int D = 128;
  const int ngroups = D / group;
  const float inv = 1.0f / (float)sqrt((double)D);
  const int n_cand = b0 * block;
  for (int g = 0; g < G; ++g) {
    for (int r = 0; r < R; ++r) {
      const int row = g * R + r;
      const float* qr = q + (int64_t)row * D;
      for (int n = 0; n < n_cand; ++n) {
        const int64_t pos = (int64_t)sink + (int64_t)pages[(int64_t)row * b0 + n / block] * block + n % block;
        const int64_t tr = (int64_t)g * entry_stride + pos;
        float part[4];
        for (int j = 0; j < 4; ++j) {
          const int gi = (32 * j) / group;
          const float s = to_f32(scale[tr * ngroups + gi], dtype);
          const float m = to_f32(minimum[tr * ngroups + gi], dtype);
          float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          for (int i = 0; i < 32; ++i) {
            const int d = 32 * j + i;
            const uint8_t byte = packed[tr * (D / 2) + d / 2];
            const uint32_t code = (d & 1) ? (byte >> 4) : (byte & 15u);
            const float kv = (float)code * s + m;
            acc[i & 3] = fmaf(kv, qr[d], acc[i & 3]);
          }
          part[j] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
        }
        const float sum = (part[0] + part[1]) + (part[2] + part[3]);
        logits[(int64_t)row * n_cand + n] = sum * inv;
      }
    }
  }
}

/* ---- top-p + GQA union ---------------------------------------------------------------------------
 * hi/twilight_exact_top_p_graph.py:19-32 and hi/twilight_offload_cache.py:1266-1310:
 * count = (number of sorted cumulative probabilities < p) + 1 = the fewest
 * largest-logit candidates whose softmax mass reaches p.  Masses here are
 * exact fixed-point integers: e = exp(l - max) by det_exp, mass = e * 2^48
 * truncated, target = ceil(sum * p).  Ties at the threshold logit are taken
 * in candidate order.  Union (hi/twilight_offload_cache.py:1527-1549, sorted
 * as np.flatnonzero at :1602-1614): [0, sink_end) U [recent_start, L) U all
 * heads' selected positions of the group. */
static double det_exp(double x) {
  if (!(x >= -700.0)) return 0.0;
  const double log2e = 1.4426950408889634;
  const double ln2 = 0.6931471805599453;
  double t = x * log2e;
  double k = floor(t + 0.5);
  double r = x + -(k * ln2);
  double p = 1.0 / 6227020800.0;
  p = p * r + 1.0 / 479001600.0;
  p = p * r + 1.0 / 39916800.0;
  p = p * r + 1.0 / 3628800.0;
  p = p * r + 1.0 / 362880.0;
  p = p * r + 1.0 / 40320.0;
  p = p * r + 1.0 / 5040.0;
  p = p * r + 1.0 / 720.0;
  p = p * r + 1.0 / 120.0;
  p = p * r + 1.0 / 24.0;
  p = p * r + 1.0 / 6.0;
  p = p * r + 0.5;
  p = p * r + 1.0;
  p = p * r + 1.0;
  uint64_t biased = (uint64_t)((int64_t)k + 1023);
  uint64_t bits = biased << 52;
  double two_k;
  memcpy(&two_k, &bits, 8);
  return p * two_k;
}

double orc_det_exp(double x) { return det_exp(x); }

static const double kMassScale = 281474976710656.0; /* 2^48 */

static unsigned long long mass_of(double e) { return (unsigned long long)(e * kMassScale); }

int orc_top_p_union(const float* logits, const int32_t* pages, int G, int R, int b0, int block,
                    int sink, double top_p, int64_t L, int64_t sink_end, int64_t recent_start,
                    int32_t* union_pos, int64_t pos_stride, int32_t* union_count,
                    int32_t* head_count, int32_t* head_pos) {
  const int n = b0 * block;
  keyed_t* buf = (keyed_t*)malloc(sizeof(keyed_t) * (size_t)(n > 0 ? n : 1));
  unsigned char* sel = (unsigned char*)malloc((size_t)(n > 0 ? n : 1));
  unsigned char* member = (unsigned char*)malloc((size_t)(L > 0 ? L : 1));
  int bad = 0;
  for (int g = 0; g < G; ++g) {
    memset(member, 0, (size_t)(L > 0 ? L : 1));
    for (int64_t p = 0; p < L; ++p)
      if (p < sink_end || p >= recent_start) member[p] = 1;
    for (int r = 0; r < R; ++r) {
      const int row = g * R + r;
      const float* lr = logits + (int64_t)row * n;
      uint32_t kmax = 0;
      for (int i = 0; i < n; ++i) {
        buf[i].key = float_key(lr[i]);
        buf[i].idx = i;
        if (buf[i].key > kmax) kmax = buf[i].key;
      }
      const float lmax = key_float(kmax);
      unsigned long long z = 0;
      for (int i = 0; i < n; ++i) z += mass_of(det_exp((double)(key_float(buf[i].key) - lmax)));
      double t = ceil((double)z * top_p);
      unsigned long long target = (t >= (double)z) ? z : (unsigned long long)t;
      if (target == 0) target = 1;
      qsort(buf, (size_t)n, sizeof(keyed_t), cmp_desc_key_asc_idx);
      unsigned long long acc = 0;
      int count = 0;
      memset(sel, 0, (size_t)n);
      for (int i = 0; i < n; ++i) {
        acc += mass_of(det_exp((double)(key_float(buf[i].key) - lmax)));
        sel[buf[i].idx] = 1;
        ++count;
        if (acc >= target) break;
      }
      head_count[row] = count;
      int slot = 0;
      for (int i = 0; i < n; ++i) {
        if (!sel[i]) continue;
        const int64_t pos = (int64_t)sink + (int64_t)pages[(int64_t)row * b0 + i / block] * block + i % block;
        if (head_pos) head_pos[(int64_t)row * n + slot] = (int32_t)pos;
        ++slot;
        if (pos < 0 || pos >= L) {
          bad = 1;
          continue;
        }
        member[pos] = 1;
      }
    }
    int32_t c = 0;
    for (int64_t p = 0; p < L; ++p)
      if (member[p]) union_pos[(int64_t)g * pos_stride + c++] = (int32_t)p;
    union_count[g] = c;
  }
  free(buf);
  free(sel);
  free(member);
  return bad;
}
