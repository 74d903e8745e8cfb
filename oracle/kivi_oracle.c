/*
 * kivi_oracle.c -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * CPU restatement of truellm-engine's KIVI quantizer and decode-attention
 * math, used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * leg to check the CUDA path.  Nothing in the shipped library links or calls
 * this file.
 *
 * What it restates (reference paths are relative to the truellm-engine tree):
 *   - kivi_compressed_bytes / kivi_params_supported
 *       src/inference/backends/cuda/compression/kivi_cache.cuh:32-43, kivi_cache.cu:205-211
 *   - kivi_compress_kernel (outlier slot algorithm + min-max INT4 groups)
 *       src/inference/backends/cuda/compression/kivi_cache.cu:23-125
 *   - kivi_decompress_kernel (fmaf dequant, fp16 output)
 *       src/inference/backends/cuda/compression/kivi_cache.cu:130-198
 *   - the per-group quantizer primitive (kivi_cache.cu:92-124), generalised to
 *     2-bit codes by replacing 15 with 3 (no reference implementation of INT2).
 *   - decode attention semantics: score = (q.k) * scale, GQA kv_head = h / (Hq/Hkv),
 *     max-subtracted softmax, out = sum p*v   (third_party/custom_kernels/megakernel.cu:267-350)
 *   - split-KV log-sum-exp merge   (third_party/vllm_kernels/paged_attention_v2.cu:132-170)
 *   - chunked-prefill attention: the same semantics per query token with a
 *     causal limit (the reference's prefill site, cuda_engine.cpp:842-860,
 *     runs it token by token)
 *
 * The paged KIVI cache format (pages, key groups per channel over G tokens,
 * value groups per token over G channels, fp16 residual ring) has no reference
 * implementation; it is restated here from the format definition in
 * include/truellm_kivi.h so that the CUDA append kernel can be checked byte for
 * byte.
 *
 * Floating point: compiled with -ffp-contract=off; the only fused multiply-add
 * is the explicit fmaf() that the reference's decompress gets from nvcc's
 * default contraction.  Division is IEEE (-prec-div=true is nvcc's default for
 * the reference TU).  fp32->fp16 is round-to-nearest-even via _Float16.
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>

/* ------------------------------------------------------------------ */
/* scalar helpers                                                      */
/* ------------------------------------------------------------------ */
float or_h2f(uint16_t h) {
  _Float16 x;
  memcpy(&x, &h, 2);
  return (float)x;
}

/* fp32 -> fp16, round to nearest even.  NaN maps to 0x7fff, the canonical
 * NaN that the GPU's cvt.rn.f16.f32 produces. */
uint16_t or_f2h(float f) {
  if (f != f) return 0x7fffu;
  _Float16 x = (_Float16)f;
  uint16_t h;
  memcpy(&h, &x, 2);
  return h;
}

static inline float bf2f(uint16_t b) {
  uint32_t u = ((uint32_t)b) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* __float2int_rn: round half to even, NaN -> 0, saturate to int range
 * (PTX cvt.rni.s32.f32 semantics). */
static inline int f2i_rn(float x) {
  if (x != x) return 0;
  if (x >= 2147483647.0f) return 2147483647;
  if (x <= -2147483648.0f) return (int)(-2147483647 - 1);
  return (int)nearbyintf(x);
}

/* ------------------------------------------------------------------ */
/* reference-format KIVI (kivi_cache.cuh / kivi_cache.cu)               */
/* ------------------------------------------------------------------ */
#define OR_KIVI_MAX_HEAD_DIM 128
#define OR_KIVI_MAX_OUTLIERS 64

/* kivi_cache.cuh:32-43 */
size_t or_kivi_compressed_bytes(int head_dim, int n_outliers, int group_size) {
  int n_res = head_dim - n_outliers;
  int n_groups = (n_res + group_size - 1) / group_size;
  return (size_t)n_outliers * 3 + (size_t)n_groups * (size_t)(group_size / 2 + 4);
}

/* kivi_cache.cu:205-211 */
int or_kivi_params_supported(int head_dim, int n_outliers, int group_size) {
  return head_dim > 0 && head_dim <= OR_KIVI_MAX_HEAD_DIM && n_outliers >= 0 &&
         n_outliers <= OR_KIVI_MAX_OUTLIERS && group_size > 0 && n_outliers <= head_dim;
}

/* The a1' primitive (kivi_cache.cu:92-124) over n fp32 values x[i*stride]:
 * sequential min/max seeded with +-FLT_MAX, degenerate when !(range > 1e-6),
 * scale = qmax/range, q = clamp(rint((x-gmin)*scale), 0, qmax),
 * stored step = 1/scale (fp16), stored zero = gmin if finite else 0 (fp16). */
void or_quant_group(const float* x, int n, int stride, int qmax, uint8_t* q, uint16_t* hscale,
                    uint16_t* hzero) {
  float gmin = FLT_MAX, gmax = -FLT_MAX;
  for (int i = 0; i < n; ++i) {
    float v = x[(size_t)i * stride];
    if (v < gmin) gmin = v;
    if (v > gmax) gmax = v;
  }
  float range = gmax - gmin;
  int degenerate = !(range > 1e-6f);
  float scale = degenerate ? 0.f : ((float)qmax / range);
  for (int i = 0; i < n; ++i) {
    float v = x[(size_t)i * stride];
    int c = f2i_rn((v - gmin) * scale);
    if (c < 0) c = 0;
    if (c > qmax) c = qmax;
    q[i] = (uint8_t)c;
  }
  float step = degenerate ? 0.f : (1.f / scale);
  int gmin_ok = (gmin == gmin) && (gmin > -FLT_MAX) && (gmin < FLT_MAX);
  *hscale = or_f2h(step);
  *hzero = or_f2h(gmin_ok ? gmin : 0.f);
}

/* kivi_compress_kernel (kivi_cache.cu:23-125), one vector at a time.
 * Bytes the reference does not write (slack of a partial last group) are
 * left untouched. */
void or_kivi_compress(const uint16_t* in, uint8_t* out, int n_vecs, int head_dim, int n_outliers,
                      int group_size) {
  if (n_vecs <= 0) return;
  if (!or_kivi_params_supported(head_dim, n_outliers, group_size)) return; /* :219-220 */
  size_t stride = or_kivi_compressed_bytes(head_dim, n_outliers, group_size);
  for (int v = 0; v < n_vecs; ++v) {
    const uint16_t* src = in + (size_t)v * head_dim;
    uint8_t* p = out + (size_t)v * stride;
    int n_out = n_outliers < OR_KIVI_MAX_OUTLIERS ? n_outliers : OR_KIVI_MAX_OUTLIERS;
    if (n_out < 0) n_out = 0;
    if (n_out > head_dim) n_out = head_dim;
    uint8_t oidx[OR_KIVI_MAX_OUTLIERS + 1];
    float omag[OR_KIVI_MAX_OUTLIERS + 1];
    for (int i = 0; i < n_out; ++i) {
      oidx[i] = 0;
      omag[i] = -1.f;
    }
    float min_mag = -1.f;
    int min_pos = 0;
    for (int d = 0; d < head_dim; ++d) {
      float a = fabsf(or_h2f(src[d]));
      if (a > min_mag) {
        /* With n_out == 0 the reference still writes slot 0 of its scratch
         * arrays; the write is never read back. */
        oidx[min_pos] = (uint8_t)d;
        omag[min_pos] = a;
        min_mag = omag[0];
        min_pos = 0;
        for (int i = 1; i < n_out; ++i)
          if (omag[i] < min_mag) {
            min_mag = omag[i];
            min_pos = i;
          }
      }
    }
    uint8_t is_out[OR_KIVI_MAX_HEAD_DIM] = {0};
    for (int i = 0; i < n_out; ++i)
      if (oidx[i] < head_dim) is_out[oidx[i]] = 1;
    for (int i = 0; i < n_out; ++i) {
      *p++ = oidx[i];
      memcpy(p, &src[oidx[i]], 2);
      p += 2;
    }
    int n_res = head_dim - n_out;
    int n_groups = (n_res + group_size - 1) / group_size;
    float res[OR_KIVI_MAX_HEAD_DIM];
    int r = 0;
    for (int d = 0; d < head_dim && r < n_res; ++d)
      if (!is_out[d]) res[r++] = or_h2f(src[d]);
    for (int g = 0; g < n_groups; ++g) {
      int gs = g * group_size, ge = gs + group_size;
      if (ge > n_res) ge = n_res;
      uint8_t q[OR_KIVI_MAX_HEAD_DIM];
      uint16_t hs, hz;
      or_quant_group(res + gs, ge - gs, 1, 15, q, &hs, &hz);
      for (int i = gs; i < ge; i += 2) {
        int q0 = q[i - gs];
        int q1 = (i + 1 < ge) ? q[i + 1 - gs] : 0;
        *p++ = (uint8_t)((q1 << 4) | q0);
      }
      memcpy(p, &hs, 2);
      p += 2;
      memcpy(p, &hz, 2);
      p += 2;
    }
  }
}

/* kivi_decompress_kernel (kivi_cache.cu:130-198). */
void or_kivi_decompress(const uint8_t* in, uint16_t* out, int n_vecs, int head_dim, int n_outliers,
                        int group_size) {
  if (n_vecs <= 0) return;
  if (!or_kivi_params_supported(head_dim, n_outliers, group_size)) return;
  size_t stride = or_kivi_compressed_bytes(head_dim, n_outliers, group_size);
  for (int v = 0; v < n_vecs; ++v) {
    const uint8_t* p = in + (size_t)v * stride;
    uint16_t* dst = out + (size_t)v * head_dim;
    int n_out = n_outliers < OR_KIVI_MAX_OUTLIERS ? n_outliers : OR_KIVI_MAX_OUTLIERS;
    if (n_out < 0) n_out = 0;
    if (n_out > head_dim) n_out = head_dim;
    float result[OR_KIVI_MAX_HEAD_DIM];
    uint8_t written[OR_KIVI_MAX_HEAD_DIM];
    memset(result, 0, sizeof(result));
    memset(written, 0, sizeof(written));
    for (int i = 0; i < n_out; ++i) {
      uint8_t ch = *p++;
      uint16_t hv;
      memcpy(&hv, p, 2);
      p += 2;
      if (ch < head_dim) {
        result[ch] = or_h2f(hv);
        written[ch] = 1;
      }
    }
    int n_res = head_dim - n_out;
    int n_groups = (n_res + group_size - 1) / group_size;
    int rch[OR_KIVI_MAX_HEAD_DIM];
    int r = 0;
    for (int d = 0; d < head_dim && r < n_res; ++d)
      if (!written[d]) rch[r++] = d;
    for (int g = 0; g < n_groups; ++g) {
      int gs = g * group_size, ge = gs + group_size;
      if (ge > n_res) ge = n_res;
      const uint8_t* pack = p;
      p += (ge - gs + 1) / 2;
      uint16_t hs, hz;
      memcpy(&hs, p, 2);
      p += 2;
      memcpy(&hz, p, 2);
      p += 2;
      float sc = or_h2f(hs), zr = or_h2f(hz);
      for (int i = gs; i < ge; ++i) {
        int bo = (i - gs) / 2;
        int nib = ((i - gs) % 2 == 0) ? (pack[bo] & 0x0f) : (pack[bo] >> 4);
        int ch = rch[i];
        if (ch >= 0 && ch < head_dim) result[ch] = fmaf((float)nib, sc, zr);
      }
    }
    for (int d = 0; d < head_dim; ++d) dst[d] = or_f2h(result[d]);
  }
}

/* ------------------------------------------------------------------ */
/* paged KIVI format (defined in include/truellm_kivi.h)               */
/* ------------------------------------------------------------------ */
typedef struct {
  int head_dim;   /* D: 64 or 128 */
  int group;      /* G: 16, 32, 64 or 128 */
  int residual;   /* R >= 0 */
  int bits;       /* 4 or 2 */
  int n_kv_heads; /* Hkv */
  int ring_cap;   /* C = round_up(R + G, 16) */
  int n_vgroups;  /* ceil(D / G) */
  int k_codes_off, v_codes_off, v_meta_off, k_meta_off, k_meta_slice;
  long page_bytes; /* bytes of one (page, kv head) block */
} or_fmt;

#define OR_PAGE 16

int or_fmt_init(or_fmt* f, int head_dim, int group, int residual, int bits, int n_kv_heads) {
  if (head_dim != 64 && head_dim != 128) return 1;
  if (group != 16 && group != 32 && group != 64 && group != 128) return 1;
  if (bits != 4 && bits != 2) return 1;
  if (residual < 0 || n_kv_heads <= 0) return 1;
  f->head_dim = head_dim;
  f->group = group;
  f->residual = residual;
  f->bits = bits;
  f->n_kv_heads = n_kv_heads;
  f->ring_cap = ((residual + group + OR_PAGE - 1) / OR_PAGE) * OR_PAGE;
  f->n_vgroups = (head_dim + group - 1) / group;
  int codes = OR_PAGE * head_dim * bits / 8;
  f->k_codes_off = 0;
  f->v_codes_off = codes;
  f->v_meta_off = 2 * codes;
  f->k_meta_off = f->v_meta_off + OR_PAGE * f->n_vgroups * 4;
  f->k_meta_slice = head_dim * 4 * OR_PAGE / group;
  long pb = f->k_meta_off + f->k_meta_slice;
  f->page_bytes = (pb + 15) / 16 * 16;
  return 0;
}

long or_fmt_page_bytes(int head_dim, int group, int residual, int bits, int n_kv_heads) {
  or_fmt f;
  if (or_fmt_init(&f, head_dim, group, residual, bits, n_kv_heads)) return -1;
  return f.page_bytes;
}

int or_nq(const or_fmt* f, int len) {
  int x = len - f->residual;
  if (x < 0) x = 0;
  return f->group * (x / f->group);
}

/* Value-code position inside a page's V block: returns the byte offset and
 * the bit shift of the code for (channel c, token t). */
static void vcode_pos(const or_fmt* f, int c, int t, int* byte_off, int* shift) {
  int mb = c / 16, cc = c % 16;
  int g = cc % 8, rh = cc / 8;
  int th = t / 8, tig = (t % 8) / 2, e = t % 2;
  int lane = g * 4 + tig;
  int W = f->head_dim * f->bits / 64; /* 32-bit words per lane */
  int VW = W < 4 ? W : 4;              /* words per vector chunk */
  int k = rh * 2 + th;                 /* register slot: R0=0,R2=1,R1=2,R3=3 -> see header */
  int w, bitpos;
  if (f->bits == 4) {
    w = mb;
    bitpos = 4 * (k + 4 * e);
  } else {
    w = mb / 2;
    bitpos = 2 * ((mb % 2) * 4 + k + 8 * e);
  }
  int word_off = ((w / VW) * 32 + lane) * (VW * 4) + (w % VW) * 4;
  *byte_off = word_off + bitpos / 8;
  *shift = bitpos % 8;
}

/* Offset (in halves) of element (token t in 0..15, channel c) inside the K or
 * V block of one 16-token residual chunk (fragment order). */
static long ring_k_off(int c, int t) {
  int kb = c / 16, cc = c % 16, hi = cc / 8, tig = (cc % 8) / 2, e = cc % 2;
  int g = t % 8, th = t / 8, lane = g * 4 + tig, r = hi * 2 + th;
  return ((long)kb * 32 + lane) * 8 + r * 2 + e;
}
static long ring_v_off(int c, int t) {
  int mb = c / 16, cc = c % 16, g = cc % 8, rh = cc / 8;
  int th = t / 8, tig = (t % 8) / 2, e = t % 2, lane = g * 4 + tig, r = th * 2 + rh;
  return ((long)mb * 32 + lane) * 8 + r * 2 + e;
}

/* Pointer (halves) to the K (kv=0) or V (kv=1) block of ring slot `slot` for (seq b, head h). */
static uint16_t* ring_chunk(const or_fmt* f, uint16_t* ring, int b, int h, int slot, int kv) {
  long chunks = f->ring_cap / OR_PAGE;
  long chunk = slot / OR_PAGE;
  long elems = (long)OR_PAGE * f->head_dim;
  return ring + ((((long)b * f->n_kv_heads + h) * chunks + chunk) * 2 + kv) * elems;
}

uint16_t or_ring_get(const or_fmt* f, const uint16_t* ring, int b, int h, int tok, int kv, int c) {
  int slot = tok % f->ring_cap;
  const uint16_t* ch = ring_chunk(f, (uint16_t*)ring, b, h, slot, kv);
  int t = slot % OR_PAGE;
  return ch[kv == 0 ? ring_k_off(c, t) : ring_v_off(c, t)];
}

static void ring_put(const or_fmt* f, uint16_t* ring, int b, int h, int tok, int kv, int c,
                     uint16_t v) {
  int slot = tok % f->ring_cap;
  uint16_t* ch = ring_chunk(f, ring, b, h, slot, kv);
  int t = slot % OR_PAGE;
  ch[kv == 0 ? ring_k_off(c, t) : ring_v_off(c, t)] = v;
}

static uint8_t* page_block(const or_fmt* f, uint8_t* pool, int phys, int h) {
  return pool + ((long)phys * f->n_kv_heads + h) * f->page_bytes;
}

/* Quantise one group of G tokens [t0, t0+G) of (seq b, head h) whose fp16
 * values are given as kx[t][c], vx[t][c] (t relative to t0), writing the
 * pages named by the block table row `bt`. */
static void pack_group(const or_fmt* f, uint8_t* pool, const int32_t* bt, int h, int t0,
                       const uint16_t* kx, const uint16_t* vx) {
  const int D = f->head_dim, G = f->group, qmax = (1 << f->bits) - 1;
  float col[128];
  uint8_t q[128];
  uint8_t kcode[128][128];
  uint16_t kmeta[128 * 2];
  /* keys: per channel over the G tokens */
  for (int c = 0; c < D; ++c) {
    for (int t = 0; t < G; ++t) col[t] = or_h2f(kx[t * D + c]);
    uint16_t hs, hz;
    or_quant_group(col, G, 1, qmax, q, &hs, &hz);
    for (int t = 0; t < G; ++t) kcode[t][c] = q[t];
    kmeta[2 * c] = hs;
    kmeta[2 * c + 1] = hz;
  }
  int pages = G / OR_PAGE;
  for (int pi = 0; pi < pages; ++pi) {
    int lp = (t0 / OR_PAGE) + pi;
    uint8_t* blk = page_block(f, pool, bt[lp], h);
    /* K codes: row-major [16][D*bits/8], lowest bits = lowest channel */
    int rb = D * f->bits / 8;
    for (int t = 0; t < OR_PAGE; ++t) {
      uint8_t* row = blk + f->k_codes_off + t * rb;
      memset(row, 0, rb);
      for (int c = 0; c < D; ++c) {
        int bitpos = c * f->bits;
        row[bitpos / 8] |= (uint8_t)(kcode[pi * OR_PAGE + t][c] << (bitpos % 8));
      }
    }
    /* K meta slice pi of the group's [D][scale, zero] array */
    memcpy(blk + f->k_meta_off, ((uint8_t*)kmeta) + (long)pi * f->k_meta_slice, f->k_meta_slice);
    /* V: per token over groups of G channels */
    memset(blk + f->v_codes_off, 0, OR_PAGE * D * f->bits / 8);
    for (int t = 0; t < OR_PAGE; ++t) {
      const uint16_t* row = vx + (long)(pi * OR_PAGE + t) * D;
      for (int vg = 0; vg < f->n_vgroups; ++vg) {
        int c0 = vg * G, c1 = c0 + G;
        if (c1 > D) c1 = D;
        for (int c = c0; c < c1; ++c) col[c - c0] = or_h2f(row[c]);
        uint16_t hs, hz;
        or_quant_group(col, c1 - c0, 1, qmax, q, &hs, &hz);
        uint16_t* vm = (uint16_t*)(blk + f->v_meta_off) + (t * f->n_vgroups + vg) * 2;
        vm[0] = hs;
        vm[1] = hz;
        for (int c = c0; c < c1; ++c) {
          int bo, sh;
          vcode_pos(f, c, t, &bo, &sh);
          blk[f->v_codes_off + bo] |= (uint8_t)(q[c - c0] << sh);
        }
      }
    }
  }
}

static uint16_t in_to_h(const uint16_t* p, int in_bf16) {
  return in_bf16 ? or_f2h(bf2f(*p)) : *p;
}

/* Append new tokens to every sequence (the quantize-on-append operation).
 *   k_new, v_new : [T_total, Hkv, D] fp16 or bf16 bits (in_bf16)
 *   cu_new       : [B+1] token offsets into k_new / v_new
 *   lens_old     : [B] context length before the append
 *   block_tables : [B, max_blocks] physical page ids (pages covering the new
 *                  length must be present)
 * Mirrors the two-phase GPU operation: first every newly complete group is
 * quantised into its pages (reading the ring for old tokens), then the new
 * residual tokens are written to the ring. */
int or_append(const or_fmt* f, uint8_t* pool, uint16_t* ring, const uint16_t* k_new,
              const uint16_t* v_new, int in_bf16, const int32_t* cu_new, const int32_t* lens_old,
              const int32_t* block_tables, int max_blocks, int B) {
  const int D = f->head_dim, G = f->group, H = f->n_kv_heads;
  uint16_t* kx = (uint16_t*)malloc(sizeof(uint16_t) * G * D);
  uint16_t* vx = (uint16_t*)malloc(sizeof(uint16_t) * G * D);
  for (int b = 0; b < B; ++b) {
    int L = lens_old[b], T = cu_new[b + 1] - cu_new[b], L2 = L + T;
    int nq0 = or_nq(f, L), nq1 = or_nq(f, L2);
    const int32_t* bt = block_tables + (long)b * max_blocks;
    for (int h = 0; h < H; ++h) {
      for (int t0 = nq0; t0 < nq1; t0 += G) {
        for (int t = 0; t < G; ++t) {
          int tok = t0 + t;
          for (int c = 0; c < D; ++c) {
            if (tok < L) {
              kx[t * D + c] = or_ring_get(f, ring, b, h, tok, 0, c);
              vx[t * D + c] = or_ring_get(f, ring, b, h, tok, 1, c);
            } else {
              long row = ((long)cu_new[b] + (tok - L)) * H + h;
              kx[t * D + c] = in_to_h(k_new + row * D + c, in_bf16);
              vx[t * D + c] = in_to_h(v_new + row * D + c, in_bf16);
            }
          }
        }
        pack_group(f, pool, bt, h, t0, kx, vx);
      }
    }
  }
  for (int b = 0; b < B; ++b) {
    int L = lens_old[b], T = cu_new[b + 1] - cu_new[b], L2 = L + T;
    int nq1 = or_nq(f, L2);
    int start = nq1 > L ? nq1 : L;
    for (int h = 0; h < H; ++h)
      for (int tok = start; tok < L2; ++tok) {
        long row = ((long)cu_new[b] + (tok - L)) * H + h;
        for (int c = 0; c < D; ++c) {
          ring_put(f, ring, b, h, tok, 0, c, in_to_h(k_new + row * D + c, in_bf16));
          ring_put(f, ring, b, h, tok, 1, c, in_to_h(v_new + row * D + c, in_bf16));
        }
      }
  }
  free(kx);
  free(vx);
  return 0;
}

/* Unpack token `tok` (< n_q) of (b, h) from the pages: canonical codes and the
 * fp16 scale/zero that apply to it.  kcode/vcode: [D]; kscale/kzero: [D]
 * (per channel, of the token's key group); vscale/vzero: [n_vgroups]. */
void or_unpack_token(const or_fmt* f, const uint8_t* pool, const int32_t* bt, int h, int tok,
                     uint8_t* kcode, uint16_t* kscale, uint16_t* kzero, uint8_t* vcode,
                     uint16_t* vscale, uint16_t* vzero) {
  const int D = f->head_dim, G = f->group;
  int lp = tok / OR_PAGE, t = tok % OR_PAGE;
  const uint8_t* blk = page_block(f, (uint8_t*)pool, bt[lp], h);
  int rb = D * f->bits / 8, mask = (1 << f->bits) - 1;
  for (int c = 0; c < D; ++c) {
    int bitpos = c * f->bits;
    kcode[c] = (blk[f->k_codes_off + t * rb + bitpos / 8] >> (bitpos % 8)) & mask;
    int bo, sh;
    vcode_pos(f, c, t, &bo, &sh);
    vcode[c] = (blk[f->v_codes_off + bo] >> sh) & mask;
  }
  /* key meta is spread over the group's pages: slice i lives in page i */
  int g0 = (tok / G) * G;
  for (int c = 0; c < D; ++c) {
    long byte = (long)c * 4;
    int pi = (int)(byte / f->k_meta_slice);
    int off = (int)(byte % f->k_meta_slice);
    const uint8_t* mb = page_block(f, (uint8_t*)pool, bt[g0 / OR_PAGE + pi], h) + f->k_meta_off;
    memcpy(&kscale[c], mb + off, 2);
    memcpy(&kzero[c], mb + off + 2, 2);
  }
  const uint16_t* vm = (const uint16_t*)(blk + f->v_meta_off) + t * f->n_vgroups * 2;
  for (int vg = 0; vg < f->n_vgroups; ++vg) {
    vscale[vg] = vm[2 * vg];
    vzero[vg] = vm[2 * vg + 1];
  }
}

/* Dequantised fp32 values (fp16-rounded, as the reference decompress writes
 * __half) of token `tok` of (b, h): from the pages when tok < n_q, else the
 * fp16 ring. */
void or_token_kv(const or_fmt* f, const uint8_t* pool, const uint16_t* ring, const int32_t* bt,
                 int b, int h, int tok, int nq, float* k, float* v) {
  const int D = f->head_dim, G = f->group;
  if (tok < nq) {
    uint8_t kc[128], vc[128];
    uint16_t ks[128], kz[128], vs[8], vz[8];
    or_unpack_token(f, pool, bt, h, tok, kc, ks, kz, vc, vs, vz);
    for (int c = 0; c < D; ++c) {
      k[c] = or_h2f(or_f2h(fmaf((float)kc[c], or_h2f(ks[c]), or_h2f(kz[c]))));
      int vg = c / G;
      v[c] = or_h2f(or_f2h(fmaf((float)vc[c], or_h2f(vs[vg]), or_h2f(vz[vg]))));
    }
  } else {
    for (int c = 0; c < D; ++c) {
      k[c] = or_h2f(or_ring_get(f, ring, b, h, tok, 0, c));
      v[c] = or_h2f(or_ring_get(f, ring, b, h, tok, 1, c));
    }
  }
}

/* Decode attention over the paged cache for tokens [tok_lo, tok_hi) of every
 * sequence (clipped to its length), in fp64.  Writes the unnormalised
 * partial state per (b, q head): m = max score (natural-log domain, scaled),
 * l = sum exp(s - m), o[D] = sum exp(s - m) * v.  An empty range gives
 * m = -inf, l = 0, o = 0.
 *   q: [B, Hq, D] fp32 values (exactly the bf16/fp16 inputs). */
typedef struct {
  const or_fmt* f;
  const uint8_t* pool;
  const uint16_t* ring;
  const float* q;
  const int32_t* block_tables;
  int max_blocks;
  const int32_t* seq_lens;
  int B, Hq;
  double scale;
  int tok_lo, tok_hi;
  double *m_out, *l_out, *o_out;
  int next; /* next (b, h) work item, taken under `mu` */
  pthread_mutex_t mu;
} decode_job;

static void decode_one(decode_job* J, int b, int h) {
  const or_fmt* f = J->f;
  const int D = f->head_dim, H = f->n_kv_heads, Hq = J->Hq, grp = Hq / H;
  int L = J->seq_lens[b];
  int lo = J->tok_lo < 0 ? 0 : J->tok_lo;
  int hi = J->tok_hi < L ? J->tok_hi : L;
  int nq = or_nq(f, L);
  const int32_t* bt = J->block_tables + (long)b * J->max_blocks;
  int n = hi > lo ? hi - lo : 0;
  double* s = (double*)malloc(sizeof(double) * (n > 0 ? n : 1) * grp);
  float* kv = (float*)malloc(sizeof(float) * 2 * D * (n > 0 ? n : 1));
  for (int i = 0; i < n; ++i)
    or_token_kv(f, J->pool, J->ring, bt, b, h, lo + i, nq, kv + (long)i * 2 * D,
                kv + (long)i * 2 * D + D);
  for (int j = 0; j < grp; ++j) {
    int hq = h * grp + j;
    const float* qq = J->q + ((long)b * Hq + hq) * D;
    double m = -INFINITY;
    for (int i = 0; i < n; ++i) {
      const float* k = kv + (long)i * 2 * D;
      double acc = 0;
      for (int c = 0; c < D; ++c) acc += (double)qq[c] * (double)k[c];
      s[(long)j * n + i] = acc * J->scale;
      if (s[(long)j * n + i] > m) m = s[(long)j * n + i];
    }
    double l = 0;
    double* o = J->o_out + ((long)b * Hq + hq) * D;
    for (int c = 0; c < D; ++c) o[c] = 0;
    for (int i = 0; i < n; ++i) {
      double p = exp(s[(long)j * n + i] - m);
      l += p;
      const float* v = kv + (long)i * 2 * D + D;
      for (int c = 0; c < D; ++c) o[c] += p * (double)v[c];
    }
    J->m_out[(long)b * Hq + hq] = m;
    J->l_out[(long)b * Hq + hq] = l;
  }
  free(s);
  free(kv);
}

static void* decode_worker(void* arg) {
  decode_job* J = (decode_job*)arg;
  int H = J->f->n_kv_heads, total = J->B * H;
  for (;;) {
    pthread_mutex_lock(&J->mu);
    int w = J->next++;
    pthread_mutex_unlock(&J->mu);
    if (w >= total) break;
    decode_one(J, w / H, w % H);
  }
  return NULL;
}

/* Decode attention over the paged cache for tokens [tok_lo, tok_hi) of every
 * sequence (clipped to its length), in fp64.  Writes the unnormalised
 * partial state per (b, q head): m = max score (natural-log domain, scaled),
 * l = sum exp(s - m), o[D] = sum exp(s - m) * v.  An empty range gives
 * m = -inf, l = 0, o = 0.  Work items (sequence, kv head) are spread over
 * n_threads POSIX threads.
 *   q: [B, Hq, D] fp32 values (exactly the bf16/fp16 inputs). */
void or_decode_partial(const or_fmt* f, const uint8_t* pool, const uint16_t* ring,
                       const float* q, const int32_t* block_tables, int max_blocks,
                       const int32_t* seq_lens, int B, int Hq, double scale, int tok_lo,
                       int tok_hi, double* m_out, double* l_out, double* o_out, int n_threads) {
  decode_job J = {f,     pool,   ring,  q,     block_tables, max_blocks, seq_lens, B,
                  Hq,    scale,  tok_lo, tok_hi, m_out,      l_out,      o_out,    0};
  pthread_mutex_init(&J.mu, NULL);
  if (n_threads < 1) n_threads = 1;
  if (n_threads > 256) n_threads = 256;
  pthread_t th[256];
  int started = 0;
  for (int i = 1; i < n_threads; ++i)
    if (pthread_create(&th[started], NULL, decode_worker, &J) == 0) ++started;
  decode_worker(&J);
  for (int i = 0; i < started; ++i) pthread_join(th[i], NULL);
  pthread_mutex_destroy(&J.mu);
}

/* Log-sum-exp merge of P partial states per (b, q head)
 * (paged_attention_v2.cu:132-170):  M = max m_p, w_p = l_p exp(m_p - M),
 * out = sum_p exp(m_p - M) o_p / sum_p w_p.  Partials laid out [P][B*Hq](*D). */
void or_merge(int P, int BH, int D, const double* m, const double* l, const double* o,
              double* out) {
  for (int i = 0; i < BH; ++i) {
    double M = -INFINITY;
    for (int p = 0; p < P; ++p)
      if (m[(long)p * BH + i] > M) M = m[(long)p * BH + i];
    double L = 0;
    for (int c = 0; c < D; ++c) out[(long)i * D + c] = 0;
    if (M == -INFINITY) continue;
    for (int p = 0; p < P; ++p) {
      double w = exp(m[(long)p * BH + i] - M);
      L += l[(long)p * BH + i] * w;
      for (int c = 0; c < D; ++c) out[(long)i * D + c] += w * o[((long)p * BH + i) * D + c];
    }
    for (int c = 0; c < D; ++c) out[(long)i * D + c] /= L;
  }
}

/* Full decode: out[B, Hq, D] in fp64. */
void or_decode(const or_fmt* f, const uint8_t* pool, const uint16_t* ring, const float* q,
               const int32_t* block_tables, int max_blocks, const int32_t* seq_lens, int B,
               int Hq, double scale, double* out, int n_threads) {
  int BH = B * Hq, D = f->head_dim;
  double* m = (double*)malloc(sizeof(double) * BH);
  double* l = (double*)malloc(sizeof(double) * BH);
  double* o = (double*)malloc(sizeof(double) * BH * D);
  or_decode_partial(f, pool, ring, q, block_tables, max_blocks, seq_lens, B, Hq, scale, 0,
                    0x7fffffff, m, l, o, n_threads);
  or_merge(1, BH, D, m, l, o, out);
  free(m);
  free(l);
  free(o);
}

/* Chunked-prefill attention over the paged cache, in fp64 (the semantics of
 * megakernel.cu:267-350 applied per query token with a causal limit).  For
 * sequence b, the n_b = cu_q[b+1] - cu_q[b] query rows q[cu_q[b] + i] are its
 * last n_b tokens, at positions p = seq_lens[b] - n_b + i, each attending to
 * the cached tokens [0, p] -- read where the cache holds them at length
 * seq_lens[b] (pages below n_q, ring above).
 *   q: [T, Hq, D] fp32; out: [T, Hq, D] fp64.  Rows of sequences whose n_b
 *   exceeds seq_lens[b] are left untouched. */
typedef struct {
  const or_fmt* f;
  const uint8_t* pool;
  const uint16_t* ring;
  const float* q;
  const int32_t* cu_q;
  const int32_t* block_tables;
  int max_blocks;
  const int32_t* seq_lens;
  int B, Hq;
  double scale;
  double* out;
  int next;
  pthread_mutex_t mu;
} prefill_job;

static void prefill_one(prefill_job* J, int b, int h) {
  const or_fmt* f = J->f;
  const int D = f->head_dim, H = f->n_kv_heads, Hq = J->Hq, grp = Hq / H;
  const int L = J->seq_lens[b], n = J->cu_q[b + 1] - J->cu_q[b];
  if (n <= 0 || n > L) return;
  const int nq = or_nq(f, L);
  const int32_t* bt = J->block_tables + (long)b * J->max_blocks;
  float* kv = (float*)malloc(sizeof(float) * 2 * D * L);
  double* s = (double*)malloc(sizeof(double) * L);
  for (int t = 0; t < L; ++t)
    or_token_kv(f, J->pool, J->ring, bt, b, h, t, nq, kv + (long)t * 2 * D,
                kv + (long)t * 2 * D + D);
  for (int i = 0; i < n; ++i) {
    const int p = L - n + i;
    for (int j = 0; j < grp; ++j) {
      const long row = (long)(J->cu_q[b] + i) * Hq + h * grp + j;
      const float* qq = J->q + row * D;
      double m = -INFINITY;
      for (int t = 0; t <= p; ++t) {
        const float* k = kv + (long)t * 2 * D;
        double acc = 0;
        for (int c = 0; c < D; ++c) acc += (double)qq[c] * (double)k[c];
        s[t] = acc * J->scale;
        if (s[t] > m) m = s[t];
      }
      double l = 0;
      double* o = J->out + row * D;
      for (int c = 0; c < D; ++c) o[c] = 0;
      for (int t = 0; t <= p; ++t) {
        const double w = exp(s[t] - m);
        l += w;
        const float* v = kv + (long)t * 2 * D + D;
        for (int c = 0; c < D; ++c) o[c] += w * (double)v[c];
      }
      for (int c = 0; c < D; ++c) o[c] /= l;
    }
  }
  free(s);
  free(kv);
}

static void* prefill_worker(void* arg) {
  prefill_job* J = (prefill_job*)arg;
  int H = J->f->n_kv_heads, total = J->B * H;
  for (;;) {
    pthread_mutex_lock(&J->mu);
    int w = J->next++;
    pthread_mutex_unlock(&J->mu);
    if (w >= total) break;
    prefill_one(J, w / H, w % H);
  }
  return NULL;
}

void or_prefill(const or_fmt* f, const uint8_t* pool, const uint16_t* ring, const float* q,
                const int32_t* cu_q, const int32_t* block_tables, int max_blocks,
                const int32_t* seq_lens, int B, int Hq, double scale, double* out,
                int n_threads) {
  prefill_job J = {f, pool, ring, q, cu_q, block_tables, max_blocks, seq_lens, B, Hq, scale,
                   out, 0};
  pthread_mutex_init(&J.mu, NULL);
  if (n_threads < 1) n_threads = 1;
  if (n_threads > 256) n_threads = 256;
  pthread_t th[256];
  int started = 0;
  for (int i = 1; i < n_threads; ++i)
    if (pthread_create(&th[started], NULL, prefill_worker, &J) == 0) ++started;
  prefill_worker(&J);
  for (int i = 0; i < started; ++i) pthread_join(th[i], NULL);
  pthread_mutex_destroy(&J.mu);
}
