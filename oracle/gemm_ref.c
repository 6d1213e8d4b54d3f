/*
 * gemm_ref.c — CPU oracle for the fp16/bf16 GEMM path. TEST INFRASTRUCTURE ONLY: nothing in the product links it;
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it, as the checker.
 *
 * Restates the arithmetic of the reference's hot path:
 *   - kernels/triton_matmul.py:67-82: acc (fp32) += A_tile · B_tile over K, then `acc.to(c dtype)` (round to nearest
 *     even) and a masked store of the M x N output;
 *   - tune/correctness.py:100-102: the ground truth `a.float() @ b.float()`, an fp32 GEMM of the fp16-rounded inputs.
 * Element (i, j) of X is read at X[i*s0 + j*s1], as the reference's kernel takes six strides
 * (kernels/triton_matmul.py:42).
 *
 * Binary16 / bfloat16 conversions are written from the IEEE 754 encodings (sign, exponent, mantissa), not taken from
 * any library.
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

float oracle_f16_to_f32(uint16_t h) {
  const uint32_t sign = (h >> 15) & 1u, ex = (h >> 10) & 0x1fu, man = h & 0x3ffu;
  float v;
  if (ex == 0) {
    v = ldexpf((float)man, -24); /* subnormal: man * 2^-24 */
  } else if (ex == 31) {
    v = man ? NAN : INFINITY;
  } else {
    v = ldexpf((float)(man | 0x400u), (int)ex - 25); /* (1024 + man) * 2^(ex - 15 - 10) */
  }
  return sign ? -v : v;
}

uint16_t oracle_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u)); /* inf / nan */
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to infinity */
  if (ax < 0x38800000u) {                                    /* below 2^-14: subnormal result */
    float v;
    memcpy(&v, &ax, 4);
    const uint32_t m = (uint32_t)nearbyintf(v * 16777216.0f); /* exact scale by 2^24, ties to even */
    return (uint16_t)(sign | m);
  }
  const uint32_t e = (ax >> 23) - 127u + 15u;
  const uint32_t m = ax & 0x7fffffu;
  uint32_t r = (e << 10) | (m >> 13);
  const uint32_t rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r += 1u; /* a carry into the exponent is still correct */
  return (uint16_t)(sign | r);
}

float oracle_bf16_to_f32(uint16_t h) {
  const uint32_t x = (uint32_t)h << 16;
  float f;
  memcpy(&f, &x, 4);
  return f;
}

uint16_t oracle_f32_to_bf16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u); /* quiet nan */
  x += 0x7fffu + ((x >> 16) & 1u);                                           /* round to nearest even */
  return (uint16_t)(x >> 16);
}

static float decode(uint16_t h, int bf16) { return bf16 ? oracle_bf16_to_f32(h) : oracle_f16_to_f32(h); }

/*
 * C32[i*N + j] = sum_k A(i,k) * B(k,j) for i < M, j < N, accumulated in increasing k.
 * acc_double = 0: fp32 multiply-add (the kernel's arithmetic); 1: double accumulation rounded once to fp32 (an
 * order-independent ground truth). Rows are split over host threads; each element's order is fixed, so the result
 * does not depend on the thread count. Returns 0, or -1 on allocation failure.
 */
typedef struct {
  const uint16_t* A;
  int64_t sam, sak;
  const float* bf;
  float* C32;
  int64_t row0, row1, N, K;
  int bf16, acc_double, err;
} gemm_job;

static void* gemm_rows(void* arg) {
  gemm_job* j = (gemm_job*)arg;
  const int64_t N = j->N, K = j->K;
  float* accf = (float*)malloc((size_t)(N > 0 ? N : 1) * sizeof(float));
  double* accd = (double*)malloc((size_t)(N > 0 ? N : 1) * sizeof(double));
  if (!accf || !accd) {
    j->err = -1;
  } else {
    for (int64_t i = j->row0; i < j->row1; ++i) {
      if (j->acc_double) {
        for (int64_t c = 0; c < N; ++c) accd[c] = 0.0;
        for (int64_t k = 0; k < K; ++k) {
          const double a = (double)decode(j->A[i * j->sam + k * j->sak], j->bf16);
          const float* brow = j->bf + k * N;
          for (int64_t c = 0; c < N; ++c) accd[c] += a * (double)brow[c];
        }
        for (int64_t c = 0; c < N; ++c) j->C32[i * N + c] = (float)accd[c];
      } else {
        for (int64_t c = 0; c < N; ++c) accf[c] = 0.0f;
        for (int64_t k = 0; k < K; ++k) {
          const float a = decode(j->A[i * j->sam + k * j->sak], j->bf16);
          const float* brow = j->bf + k * N;
          for (int64_t c = 0; c < N; ++c) accf[c] = fmaf(a, brow[c], accf[c]);
        }
        memcpy(j->C32 + i * N, accf, (size_t)N * sizeof(float));
      }
    }
  }
  free(accf);
  free(accd);
  return NULL;
}

int oracle_gemm_f32(const uint16_t* A, int64_t sam, int64_t sak, const uint16_t* B, int64_t sbk, int64_t sbn,
                    float* C32, int64_t M, int64_t N, int64_t K, int bf16, int acc_double) {
  float* bf = (float*)malloc((size_t)(K > 0 ? K : 1) * (size_t)(N > 0 ? N : 1) * sizeof(float));
  if (!bf) return -1;
  for (int64_t k = 0; k < K; ++k)
    for (int64_t c = 0; c < N; ++c) bf[k * N + c] = decode(B[k * sbk + c * sbn], bf16);
  long nt = sysconf(_SC_NPROCESSORS_ONLN);
  if (nt < 1) nt = 1;
  if (nt > 64) nt = 64;
  if ((int64_t)nt > M) nt = M > 0 ? (long)M : 1;
  gemm_job jobs[64];
  pthread_t tids[64];
  int started[64] = {0};
  for (long t = 0; t < nt; ++t) {
    jobs[t] = (gemm_job){A, sam, sak, bf, C32, M * t / nt, M * (t + 1) / nt, N, K, bf16, acc_double, 0};
    started[t] = (t > 0) && pthread_create(&tids[t], NULL, gemm_rows, &jobs[t]) == 0;
  }
  gemm_rows(&jobs[0]);
  for (long t = 1; t < nt; ++t) {
    if (started[t]) pthread_join(tids[t], NULL);
    else gemm_rows(&jobs[t]);
  }
  int err = 0;
  for (long t = 0; t < nt; ++t) err |= jobs[t].err;
  free(bf);
  return err ? -1 : 0;
}

/* out[i] = round-to-nearest-even of x[i] into fp16 (bf16 = 0) or bf16 (bf16 = 1): the epilogue's cast
   (kernels/triton_matmul.py:82). */
void oracle_round(const float* x, uint16_t* out, int64_t n, int bf16) {
  for (int64_t i = 0; i < n; ++i) out[i] = bf16 ? oracle_f32_to_bf16(x[i]) : oracle_f32_to_f16(x[i]);
}

/* Deterministic split-K reduction restated (kernels/triton_matmul.py:85-92): out[i] = cast(sum_{s<split} ws[s*MN+i]),
   summed in increasing s in fp32. */
void oracle_splitk_reduce(const float* ws, uint16_t* out, int64_t MN, int32_t split, int bf16) {
  for (int64_t i = 0; i < MN; ++i) {
    float acc = 0.0f;
    for (int32_t s = 0; s < split; ++s) acc += ws[(int64_t)s * MN + i];
    out[i] = bf16 ? oracle_f32_to_bf16(acc) : oracle_f32_to_f16(acc);
  }
}
