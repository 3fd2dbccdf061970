/*
 * oracle_kv.c -- plain C + OpenMP restatement of MServe's KV selection-and-offload path.
 *
 * TEST INFRASTRUCTURE ONLY: the timed CPU baseline of bench.py (cpu_baseline leg and the
 * --impl reference arm) and a second oracle for the tests.  Not part of the product.
 *
 *   okv_gather      out[b,h,s,:] = in[b,h,idx[...s],:]           -- the gather semantics of
 *                   torch.index_select(k_cpu, dim=2, index) in CPUKVCache.get_sparse_async
 *                   (qwen-eljrte/Qwen_Transformer/kv_cache.py:597-599) and of the UVA
 *                   kernel (qwen-eljrte/cuda_uva_kernel.cpp:29-44), per-segment lists.
 *   okv_score_bf16  s[b,hk,t] = sum_g q[b,hk*G+g,:] . k[b,hk,t,:]  -- the per-head q_last·Kᵀ
 *                   products of compute_token_importance (attention.py:556-562) summed over
 *                   the query heads of KV head hk, fp32.
 *   okv_topk        top-k of [0, L-R) by (key desc, index asc) plus the window [L-R, L),
 *                   ascending -- the selection of attention.py:567-572 with the recent window.
 *   okv_attention_bf16  softmax(q·K_selᵀ/sqrt(D))·V_sel per KV-head group, fp32
 *                   (sparse_sdpa_attention, attention.py:619-636).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float bf16f(uint16_t x) {
  union { uint32_t u; float f; } c;
  c.u = (uint32_t)x << 16;
  return c.f;
}

static inline uint32_t order_key(float f) {
  union { float f; uint32_t u; } c;
  c.f = f;
  if ((c.u & 0x7fffffffu) > 0x7f800000u) return 0xffffffffu; /* every NaN ranks highest */
  return (c.u & 0x80000000u) ? ~c.u : (c.u | 0x80000000u);
}

int okv_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Row gather.  Strides in bytes (src) / elements (idx).  counts may be NULL. */
void okv_gather(const uint8_t* src_k, const uint8_t* src_v, int64_t sb, int64_t sh, int64_t st, int B, int H,
                const void* idx, int idx_bits, int64_t isb, int64_t ish, int S, const int32_t* counts,
                uint8_t* dst_k, uint8_t* dst_v, int64_t row_bytes, int nthreads) {
  const int64_t nseg = (int64_t)B * H;
#pragma omp parallel for schedule(static) num_threads(nthreads)
  for (int64_t seg = 0; seg < nseg; ++seg) {
    const int b = (int)(seg / H), h = (int)(seg % H);
    const int n = counts ? counts[seg] : S;
    const int64_t io = (int64_t)b * isb + (int64_t)h * ish;
    const uint8_t* sk = src_k + (int64_t)b * sb + (int64_t)h * sh;
    const uint8_t* sv = src_v + (int64_t)b * sb + (int64_t)h * sh;
    uint8_t* dk = dst_k + seg * (int64_t)S * row_bytes;
    uint8_t* dv = dst_v + seg * (int64_t)S * row_bytes;
    for (int s = 0; s < n; ++s) {
      const int64_t t = idx_bits == 64 ? ((const int64_t*)idx)[io + s] : ((const int32_t*)idx)[io + s];
      memcpy(dk + (int64_t)s * row_bytes, sk + t * st, (size_t)row_bytes);
      memcpy(dv + (int64_t)s * row_bytes, sv + t * st, (size_t)row_bytes);
    }
  }
}

/* fp32 GQA-summed scores; k strides in elements. */
void okv_score_bf16(const uint16_t* q, const uint16_t* k, int64_t k_sb, int64_t k_sh, int64_t k_st, int B, int Hq,
                    int Hkv, int T, int D, float* out, int64_t out_stride, int nthreads) {
  const int G = Hq / Hkv;
  const int64_t nseg = (int64_t)B * Hkv;
  const int64_t chunk = 256;
  const int64_t nchunks = (T + chunk - 1) / chunk;
#pragma omp parallel for schedule(static) num_threads(nthreads)
  for (int64_t w = 0; w < nseg * nchunks; ++w) {
    const int64_t seg = w / nchunks;
    const int64_t t0 = (w % nchunks) * chunk;
    const int b = (int)(seg / Hkv), h = (int)(seg % Hkv);
    float qs[1024];
    for (int d = 0; d < D; ++d) {
      float a = 0.f;
      for (int g = 0; g < G; ++g) a += bf16f(q[((int64_t)b * Hq + h * G + g) * D + d]);
      qs[d] = a;
    }
    const int64_t t1 = t0 + chunk < T ? t0 + chunk : T;
    for (int64_t t = t0; t < t1; ++t) {
      const uint16_t* row = k + (int64_t)b * k_sb + (int64_t)h * k_sh + t * k_st;
      float acc = 0.f;
      for (int d = 0; d < D; ++d) acc += qs[d] * bf16f(row[d]);
      out[seg * out_stride + t] = acc;
    }
  }
}

/* One selection: radix select of the K-th key (8-bit digits), ordered compaction. */
static int select_one(const float* row, int n, int K, int R, int L, int32_t* out, uint32_t* keys) {
  if (K > n) K = n;
  if (K < 0) K = 0;
  int pos = 0;
  if (K == n) {
    for (int t = 0; t < n; ++t) out[pos++] = t;
  } else if (K > 0) {
    for (int t = 0; t < n; ++t) keys[t] = order_key(row[t]);
    uint32_t prefix = 0, mask = 0, krem = (uint32_t)K;
    for (int shift = 24; shift >= 0; shift -= 8) {
      uint32_t hist[256] = {0};
      for (int t = 0; t < n; ++t)
        if ((keys[t] & mask) == prefix) hist[(keys[t] >> shift) & 255u]++;
      uint32_t cum = 0;
      for (int d = 255; d >= 0; --d) {
        if (cum + hist[d] >= krem) {
          prefix |= (uint32_t)d << shift;
          krem -= cum;
          break;
        }
        cum += hist[d];
      }
      mask |= 0xffu << shift;
    }
    uint32_t eq_taken = 0;
    for (int t = 0; t < n; ++t) {
      if (keys[t] > prefix) out[pos++] = t;
      else if (keys[t] == prefix && eq_taken < krem) { out[pos++] = t; ++eq_taken; }
    }
  }
  for (int t = n; t < L; ++t) out[pos++] = t;
  return pos;
}

void okv_topk(const float* scores, int64_t stride, int nsel, int sel_per_batch, const int32_t* lens, int L_scalar,
              int K, int R, int32_t* out, int64_t out_stride, int32_t* counts, int nthreads) {
#pragma omp parallel num_threads(nthreads)
  {
    uint32_t* keys = NULL;
    int cap = 0;
#pragma omp for schedule(dynamic, 1)
    for (int j = 0; j < nsel; ++j) {
      const int L = lens ? lens[j / sel_per_batch] : L_scalar;
      const int n = L > R ? L - R : 0;
      if (n > cap) {
        free(keys);
        keys = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)n);
        cap = n;
      }
      counts[j] = select_one(scores + (int64_t)j * stride, n, K, R, L, out + (int64_t)j * out_stride, keys);
    }
    free(keys);
  }
}

/* q [B,Hq,D], k_sel/v_sel [B,Hkv,S,D] (bf16), out fp32 [B,Hq,D]. */
void okv_attention_bf16(const uint16_t* q, const uint16_t* k_sel, const uint16_t* v_sel, const int32_t* counts,
                        int B, int Hq, int Hkv, int S, int D, float scale, float* out, int nthreads) {
  const int G = Hq / Hkv;
#pragma omp parallel for schedule(static) num_threads(nthreads)
  for (int64_t r = 0; r < (int64_t)B * Hq; ++r) {
    const int b = (int)(r / Hq), hq = (int)(r % Hq), hk = hq / G;
    const int64_t seg = (int64_t)b * Hkv + hk;
    const int n = counts ? counts[seg] : S;
    float qf[1024], acc[1024];
    for (int d = 0; d < D; ++d) { qf[d] = bf16f(q[r * D + d]) * scale; acc[d] = 0.f; }
    float m = -INFINITY, l = 0.f;
    for (int s = 0; s < n; ++s) {
      const uint16_t* kr = k_sel + (seg * S + s) * D;
      const uint16_t* vr = v_sel + (seg * S + s) * D;
      float dot = 0.f;
      for (int d = 0; d < D; ++d) dot += qf[d] * bf16f(kr[d]);
      const float mn = dot > m ? dot : m;
      const float corr = expf(m - mn), p = expf(dot - mn);
      l = l * corr + p;
      for (int d = 0; d < D; ++d) acc[d] = acc[d] * corr + p * bf16f(vr[d]);
      m = mn;
    }
    for (int d = 0; d < D; ++d) out[r * D + d] = l > 0.f ? acc[d] / l : 0.f;
  }
}
