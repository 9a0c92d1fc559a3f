/*
 * TEST INFRASTRUCTURE ONLY: CPU oracle for tread's chunk-reuse hot path.
 *
 * This file restates, in plain C, the arithmetic of the reference's hot path so that the
 * CUDA kernels of tread_b200 can be checked on the same inputs. It is the parity checker
 * (and, in bench.py, the timed CPU baseline), never part of the product. It is pinned
 * against golden vectors produced by the reference itself (tests/golden/make_golden.py).
 *
 * Element types: code 0 = fp32, 1 = fp16, 2 = bf16 (matches include/tread_b200.h).
 * All arithmetic is fp32 with contraction disabled (-ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- element conversions (IEEE round-to-nearest-even) -------------------------------- */

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float load_elem(const void* base, size_t i, int dtype) {
  switch (dtype) {
    case 2: return bf16_to_f32(((const uint16_t*)base)[i]);
    case 1: return (float)((const _Float16*)base)[i];
    default: return ((const float*)base)[i];
  }
}

static inline void store_elem(void* base, size_t i, float x, int dtype) {
  switch (dtype) {
    case 2: ((uint16_t*)base)[i] = f32_to_bf16(x); break;
    case 1: ((_Float16*)base)[i] = (_Float16)x; break;
    default: ((float*)base)[i] = x; break;
  }
}

static inline size_t elem_size(int dtype) { return dtype == 0 ? 4 : 2; }

/* ---- RoPE re-rotation (tread/blend.py:22-39) ------------------------------------------ */

/*
 * cos/sin of the shift `delta` for the D/2 frequencies, as HF's rotary_emb computes them in
 * fp32 (transformers Qwen2RotaryEmbedding.forward: freqs = inv_freq @ pos, emb = cat(freqs,
 * freqs), cos = emb.cos() * attention_scaling), then divided by attention_scaling as
 * rotate_keys does (tread/blend.py:36-38).
 */
void oracle_rope_cos_sin(int64_t delta, const float* inv_freq, int half, float scale, float* c,
                         float* s) {
  for (int i = 0; i < half; ++i) {
    const float a = (float)delta * inv_freq[i];
    c[i] = (cosf(a) * scale) / scale;
    s[i] = (sinf(a) * scale) / scale;
  }
}

/*
 * rotate_keys + torch.cat (tread/engine.py:108-120): segment j is a block K/V laid out
 * [L*Hkv, n_j, D]; it is rotated by delta[j] (K only, V copied) and written at token rows
 * dst0[j].. of out_k/out_v ([L*Hkv, T_out, D]). in_dtype/out_dtype pick element types;
 * out_dtype 0 with a bf16 input gives the "fp32 rotation" of the reference.
 * K' = K*cos + rotate_half(K)*sin, evaluated as fl(fl(x1*c) - fl(x2*s)) for the first half
 * and fl(fl(x2*c) + fl(x1*s)) for the second, the order torch uses for that expression.
 */
void oracle_rope_gather_append(const void* const* k_src, const void* const* v_src,
                               const int32_t* n_tok, const int64_t* delta, const int64_t* dst0,
                               int nseg, void* out_k, void* out_v, int LH, int D, int64_t T_out,
                               const float* inv_freq, float scale, int in_dtype, int out_dtype,
                               int nthreads) {
  const int half = D / 2;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#endif
  for (int j = 0; j < nseg; ++j) {
    const int n = n_tok[j];
    float* c = (float*)malloc(sizeof(float) * (size_t)half);
    float* s = (float*)malloc(sizeof(float) * (size_t)half);
    oracle_rope_cos_sin(delta[j], inv_freq, half, scale, c, s);
    const int rot = delta[j] != 0;
#pragma omp parallel for schedule(static)
    for (int lh = 0; lh < LH; ++lh) {
      for (int t = 0; t < n; ++t) {
        const size_t src = ((size_t)lh * n + t) * D;
        const size_t dst = ((size_t)lh * T_out + dst0[j] + t) * D;
        for (int i = 0; i < half; ++i) {
          const float x1 = load_elem(k_src[j], src + i, in_dtype);
          const float x2 = load_elem(k_src[j], src + half + i, in_dtype);
          float o1 = x1, o2 = x2;
          if (rot) {
            const float a = x1 * c[i], b = x2 * s[i];
            o1 = a - b;
            const float d = x2 * c[i], e = x1 * s[i];
            o2 = d + e;
          }
          store_elem(out_k, dst + i, o1, out_dtype);
          store_elem(out_k, dst + half + i, o2, out_dtype);
        }
        if (in_dtype == out_dtype) {
          memcpy((char*)out_v + dst * elem_size(out_dtype), (const char*)v_src[j] + src * elem_size(in_dtype),
                 (size_t)D * elem_size(in_dtype));
        } else {
          for (int i = 0; i < D; ++i)
            store_elem(out_v, dst + i, load_elem(v_src[j], src + i, in_dtype), out_dtype);
        }
      }
    }
    free(c);
    free(s);
  }
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ---- A4: layer-1 deviation (tread/blend.py:129) ---------------------------------------- */

/*
 * L2 norm of (x - y) over one D-row in the fixed order the CUDA kernel uses: 32 lanes own
 * E = D/32 consecutive elements each and accumulate fl(p + fl(d*d)) in element order; the
 * lane partials are combined by an xor butterfly with offsets 16, 8, 4, 2, 1; then sqrt.
 */
static float row_norm(const void* x, size_t xo, const void* y, size_t yo, int D, int dtype) {
  const int E = D / 32;
  float p[32], q[32];
  for (int l = 0; l < 32; ++l) {
    float acc = 0.f;
    for (int e = 0; e < E; ++e) {
      const float d = load_elem(x, xo + (size_t)l * E + e, dtype) - load_elem(y, yo + (size_t)l * E + e, dtype);
      const float sq = d * d;
      acc = acc + sq;
    }
    p[l] = acc;
  }
  for (int off = 16; off >= 1; off >>= 1) {
    for (int l = 0; l < 32; ++l) q[l] = p[l] + p[l ^ off];
    memcpy(p, q, sizeof(p));
  }
  return sqrtf(p[0]);
}

/*
 * dev[t] = sum_h ||k1[h,t] - K1[h,pos_t]|| + sum_h ||v1[h,t] - V1[h,pos_t]||, heads summed in
 * order, K sum + V sum last. Element (h, t, d) of the fresh rows is at t*f_st + h*f_sh + d,
 * element (h, pos, d) of the cache at pos*c_st + h*c_sh + d.
 */
void oracle_deviation(const void* k1, const void* v1, int64_t f_st, int64_t f_sh, const void* K1, const void* V1,
                      int64_t c_st, int64_t c_sh, const int64_t* cand_pos, int n, int H, int D, int dtype,
                      float* dev) {
  for (int t = 0; t < n; ++t) {
    const int64_t pos = cand_pos[t];
    float a = 0.f, b = 0.f;
    for (int h = 0; h < H; ++h) {
      const size_t fo = (size_t)(t * f_st + h * f_sh), co = (size_t)(pos * c_st + h * c_sh);
      a = a + row_norm(k1, fo, K1, co, D, dtype);
      b = b + row_norm(v1, fo, V1, co, D, dtype);
    }
    dev[t] = a + b;
  }
}
