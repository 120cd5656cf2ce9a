/*
 * TEST INFRASTRUCTURE ONLY - never linked into or called by the product library.
 *
 * CPU restatement of the arithmetic of gtx16_fp16's CUDA kernels (reference file
 * src/gtx16_fp16/kernels.py) and of the host dispatch in src/gtx16_fp16/ops.py, used by tests/,
 * __graft_entry__.smoke() and bench.py's CPU baseline leg as the checker. Each function names the
 * reference lines it follows. fp16 values are passed as raw IEEE binary16 bit patterns (uint16_t).
 *
 * Exactness: the reference's packed-fp16 FMA (__hfma2, one rounding) is emulated exactly: the
 * product of two fp16 values is exact in double, the sum is formed with round-to-odd in double
 * (TwoSum + sticky bit), and the final rounding to fp16 is round-to-nearest-even. Round-to-odd at
 * 53 bits followed by RNE at 11 bits equals a single RNE rounding of the exact value.
 * fp32 FMAs use C99 fmaf (single rounding), matching the FFMA the reference compiles to with nvcc's
 * default FMA contraction (kernels.py:186-188 under --use_fast_math).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------------------------ */
/* binary16 <-> binary32/64                                                                     */
/* ------------------------------------------------------------------------------------------ */
float g16o_h2f(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1Fu;
  const uint32_t m = h & 0x3FFu;
  float v;
  if (e == 0) {
    v = ldexpf((float)m, -24); /* zero or subnormal: m * 2^-24 */
  } else if (e == 31) {
    v = m ? NAN : INFINITY;
  } else {
    v = ldexpf((float)(m | 0x400u), (int)e - 25);
  }
  uint32_t bits;
  memcpy(&bits, &v, 4);
  bits |= sign;
  memcpy(&v, &bits, 4);
  return v;
}

/* Round a double to the nearest binary16 (ties to even), with overflow to infinity. */
uint16_t g16o_d2h(double d) {
  uint16_t sign = signbit(d) ? 0x8000u : 0u;
  if (isnan(d)) return (uint16_t)(sign | 0x7E00u);
  double a = fabs(d);
  if (a >= 65520.0) return (uint16_t)(sign | 0x7C00u); /* 65504 + half an ulp ties to 2^16 */
  if (a == 0.0) return sign;
  int E;
  frexp(a, &E);                   /* a in [2^(E-1), 2^E) */
  int ue = E - 1;                 /* unbiased exponent of a */
  double quantum = ue < -14 ? ldexp(1.0, -24) : ldexp(1.0, ue - 10);
  double r = nearbyint(a / quantum) * quantum; /* exact scaling; RNE in the default mode */
  if (r >= 65520.0) return (uint16_t)(sign | 0x7C00u);
  if (r < ldexp(1.0, -14)) {
    return (uint16_t)(sign | (uint16_t)(r / ldexp(1.0, -24))); /* subnormal (or 0) */
  }
  frexp(r, &E);
  ue = E - 1;
  uint32_t mant = (uint32_t)(ldexp(r, -ue) * 1024.0) - 1024u;
  return (uint16_t)(sign | (uint16_t)((ue + 15) << 10) | (uint16_t)mant);
}

uint16_t g16o_f2h(float f) { return g16o_d2h((double)f); }

/* Exact fp16 fused multiply-add: RNE16(a*b + c). */
static uint16_t hfma(uint16_t a, uint16_t b, uint16_t c) {
  const double p = (double)g16o_h2f(a) * (double)g16o_h2f(b); /* exact: 11+11 bits */
  const double q = (double)g16o_h2f(c);
  if (!isfinite(p) || !isfinite(q)) return g16o_d2h(p + q);
  double s = p + q;
  const double bb = s - p;
  const double err = (p - (s - bb)) + (q - bb); /* TwoSum: exact error of s */
  if (err != 0.0) {
    uint64_t bits;
    memcpy(&bits, &s, 8);
    if ((bits & 1u) == 0u) { /* round to odd: move to the odd neighbour on the side of err */
      s = nextafter(s, err > 0.0 ? INFINITY : -INFINITY);
    }
  }
  return g16o_d2h(s);
}

/* ------------------------------------------------------------------------------------------ */
/* rowscale (kernels.py:227-250)                                                                */
/* ------------------------------------------------------------------------------------------ */
/* S = 2^ceil(log2(amax / thresh)) if amax > thresh else 1, exact (the reference evaluates the
 * same expression with fast-math log2f/exp2f, kernels.py:242). Returns S, writes 1/S. */
static float row_scale(float amax, float thresh, float* inv) {
  if (!(amax > thresh)) {
    *inv = 1.f;
    return 1.f;
  }
  const float r = amax / thresh;
  if (isinf(r)) {
    *inv = 0.f;
    return INFINITY;
  }
  int E;
  const float m = frexpf(r, &E); /* r = m * 2^E, m in [0.5, 1) */
  const int c = (m == 0.5f) ? E - 1 : E;
  *inv = ldexpf(1.f, -c);
  return ldexpf(1.f, c);
}

/* x_is_f16 selects rowscale_f16 (x is uint16 bits) or rowscale_f32. */
void g16o_rowscale(const void* x, int x_is_f16, uint16_t* y, float* S, int M, int K, float thresh) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < M; ++r) {
    float amax = 0.f;
    for (int k = 0; k < K; ++k) {
      const float v = x_is_f16 ? g16o_h2f(((const uint16_t*)x)[(size_t)r * K + k]) : ((const float*)x)[(size_t)r * K + k];
      amax = fmaxf(amax, fabsf(v)); /* fmaxf ignores NaN, like the kernel's fmaxf (kernels.py:234) */
    }
    float inv;
    const float sc = row_scale(amax, thresh, &inv);
    for (int k = 0; k < K; ++k) {
      const float v = x_is_f16 ? g16o_h2f(((const uint16_t*)x)[(size_t)r * K + k]) : ((const float*)x)[(size_t)r * K + k];
      y[(size_t)r * K + k] = g16o_f2h(v * inv); /* kernels.py:244 */
    }
    S[r] = sc; /* kernels.py:245 */
  }
}

/* ------------------------------------------------------------------------------------------ */
/* Hybrid-accumulation GEMM (kernels.py:35-137)                                                 */
/* ------------------------------------------------------------------------------------------ */
/* accf[M,N] = sum over 16-wide K slices of fp32(fp16 FMA chain over the slice), for the K range
 * [k0, k0 + klen): the per-thread arithmetic of hgemm_body (kernels.py:77-104). Slices start at
 * k0 and are zero-padded past klen (kernels.py:65,70), which leaves the fp16 chain unchanged. */
void g16o_hgemm_accf(const uint16_t* A, const uint16_t* B, int M, int N, int K, int k0, int klen, float* accf) {
#pragma omp parallel for schedule(dynamic, 4)
  for (int r = 0; r < M; ++r) {
    uint16_t* col_acc = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)N);
    float* row = accf + (size_t)r * N;
    for (int n = 0; n < N; ++n) row[n] = 0.f;
    for (int s0 = 0; s0 < klen; s0 += 16) {
      for (int n = 0; n < N; ++n) col_acc[n] = 0; /* __float2half2_rn(0.f), kernels.py:99 */
      const int s1 = s0 + 16 < klen ? s0 + 16 : klen;
      for (int k = s0; k < s1; ++k) {
        const uint16_t a = A[(size_t)r * K + k0 + k];
        const uint16_t* brow = B + (size_t)(k0 + k) * N;
        for (int n = 0; n < N; ++n) col_acc[n] = hfma(a, brow[n], col_acc[n]); /* kernels.py:89 */
      }
      for (int n = 0; n < N; ++n) row[n] += g16o_h2f(col_acc[n]); /* fold, kernels.py:96-98 */
    }
    free(col_acc);
  }
}

/* hgemm_f32out / hgemm_f16out epilogue (kernels.py:106-135): out = accf * rscale[row] + bias[col]. */
void g16o_hgemm(const uint16_t* A, const uint16_t* B, void* out, int out_is_f16, const float* bias, const float* rscale,
                int M, int N, int K) {
  float* accf = (float*)malloc(sizeof(float) * (size_t)M * N);
  g16o_hgemm_accf(A, B, M, N, K, 0, K, accf);
#pragma omp parallel for schedule(static)
  for (int r = 0; r < M; ++r) {
    const float rs = rscale ? rscale[r] : 1.f;
    for (int n = 0; n < N; ++n) {
      const float v = accf[(size_t)r * N + n] * rs + (bias ? bias[n] : 0.f);
      if (out_is_f16)
        ((uint16_t*)out)[(size_t)r * N + n] = g16o_f2h(v);
      else
        ((float*)out)[(size_t)r * N + n] = v;
    }
  }
  free(accf);
}

/* hgemm_splitk (kernels.py:143-147, host ops.py:92-101): C (fp32) = prefill(bias or 0) plus each K
 * chunk's accf * rscale[row]. The reference adds chunks with fp32 atomics in an arbitrary order;
 * this restatement adds them in ascending chunk order. */
void g16o_hgemm_splitk(const uint16_t* A, const uint16_t* B, float* C, const float* bias, const float* rscale, int M,
                       int N, int K, int kchunk) {
  float* accf = (float*)malloc(sizeof(float) * (size_t)M * N);
  for (int r = 0; r < M; ++r)
    for (int n = 0; n < N; ++n) C[(size_t)r * N + n] = bias ? bias[n] : 0.f; /* _prefilled, ops.py:54-62 */
  for (int kb = 0; kb < K; kb += kchunk) {
    const int klen = K - kb < kchunk ? K - kb : kchunk;
    g16o_hgemm_accf(A, B, M, N, K, kb, klen, accf);
    for (int r = 0; r < M; ++r) {
      const float rs = rscale ? rscale[r] : 1.f;
      for (int n = 0; n < N; ++n) C[(size_t)r * N + n] += accf[(size_t)r * N + n] * rs;
    }
  }
  free(accf);
}

/* ------------------------------------------------------------------------------------------ */
/* Skinny GEMM (kernels.py:163-211)                                                             */
/* ------------------------------------------------------------------------------------------ */
/* C (fp32, [M,N]) = sum over K chunks (blockIdx.y) of: sum_{t=0..7} (fp32 FMA chain over rows
 * k = kb+t, kb+t+8, ...) (+ bias in chunk 0). Chunks are added in ascending order (the reference
 * uses atomics, kernels.py:206). */
void g16o_skinny(const void* X, int x_is_f16, const uint16_t* W, const float* bias, float* C, int M, int N, int K,
                 int kchunk) {
  const int nchunks = kchunk > 0 ? (K + kchunk - 1) / kchunk : 0;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n) {
    for (int m = 0; m < M; ++m) {
      float c = 0.f; /* torch.zeros output, ops.py:79 */
      for (int y = 0; y < nchunks; ++y) {
        const int kb = y * kchunk;
        const int ke = K < kb + kchunk ? K : kb + kchunk;
        float s = 0.f;
        for (int t = 0; t < 8; ++t) {
          float acc = 0.f;
          for (int k = kb + t; k < ke; k += 8) {
            const float a = x_is_f16 ? g16o_h2f(((const uint16_t*)X)[(size_t)m * K + k]) : ((const float*)X)[(size_t)m * K + k];
            acc = fmaf(a, g16o_h2f(W[(size_t)k * N + n]), acc);
          }
          s += acc; /* smem reduce, kernels.py:202-204 */
        }
        if (bias && y == 0) s += bias[n]; /* kernels.py:205 */
        c += s;                           /* kernels.py:206 */
      }
      C[(size_t)m * N + n] = c;
    }
  }
}

/* skinny_config (ops.py:45-51): returns kchunk, writes nbx and ksplit. */
int g16o_skinny_config(int N, int K, int sms, int* nbx, int* ksplit) {
  *nbx = (N + 255) / 256;
  int ks = (4 * sms + *nbx - 1) / *nbx;
  if (K / 64 < ks) ks = K / 64;
  if (ks < 1) ks = 1;
  int kchunk = ((K + ks - 1) / ks + 7) / 8 * 8;
  *ksplit = kchunk > 0 ? (K + kchunk - 1) / kchunk : 0;
  return kchunk;
}

/* ------------------------------------------------------------------------------------------ */
/* mm_t dispatch (ops.py:65-108)                                                                */
/* ------------------------------------------------------------------------------------------ */
/* out = x @ w + bias following the reference's three-way dispatch on a GPU with `sms` SMs.
 * ROW_SCALE_THRESHOLD = 1024 (ops.py:16), SKINNY_MAX_M = 8 (kernels.py:253). */
void g16o_mm_t(const void* x, int x_is_f16, const uint16_t* w, const float* bias, void* out, int out_is_f16, int M,
               int K, int N, int sms) {
  if (M <= 8) {
    float* C = (float*)malloc(sizeof(float) * (size_t)M * N);
    int nbx, ksplit;
    const int kchunk = g16o_skinny_config(N, K, sms, &nbx, &ksplit);
    g16o_skinny(x, x_is_f16, w, bias, C, M, N, K, kchunk);
    for (size_t i = 0; i < (size_t)M * N; ++i) {
      if (out_is_f16)
        ((uint16_t*)out)[i] = g16o_f2h(C[i]); /* out.to(fp16), ops.py:84 */
      else
        ((float*)out)[i] = C[i];
    }
    free(C);
    return;
  }
  uint16_t* x16 = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)M * K);
  float* rs = (float*)malloc(sizeof(float) * (size_t)M);
  g16o_rowscale(x, x_is_f16, x16, rs, M, K, 1024.0f);
  const int tiles = ((N + 127) / 128) * ((M + 127) / 128);
  if (tiles < 2 * sms && K >= 256) {
    int ksplit = (2 * sms + tiles - 1) / tiles;
    if (K / 128 < ksplit) ksplit = K / 128;
    const int kchunk = ((K + ksplit - 1) / ksplit + 15) / 16 * 16;
    float* C = (float*)malloc(sizeof(float) * (size_t)M * N);
    g16o_hgemm_splitk(x16, w, C, bias, rs, M, N, K, kchunk);
    for (size_t i = 0; i < (size_t)M * N; ++i) {
      if (out_is_f16)
        ((uint16_t*)out)[i] = g16o_f2h(C[i]);
      else
        ((float*)out)[i] = C[i];
    }
    free(C);
  } else {
    g16o_hgemm(x16, w, out, out_is_f16, bias, rs, M, N, K);
  }
  free(x16);
  free(rs);
}

int g16o_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
