/*
 * attn_oracle.c -- TEST INFRASTRUCTURE ONLY.  CPU restatement of the
 * attention hot path of CudaTransformer, used as the parity checker by
 * tests/, by __graft_entry__.smoke() and by bench.py's CPU-baseline leg.
 * Nothing in the product (libctfa_b200.so, cudatransformer_b200/) links,
 * imports or calls this file.
 *
 * Three groups of functions, all on row-major [BH][T][D] buffers:
 *
 *  1. oracle_attention_{forward,backward}_f64: exact attention in float64
 *     (the arbiter named by the spec).  Math of the reference kernels,
 *     cuda_transformer/flash_attention.cu:6-40 (forward) and :172-187
 *     (backward): O = softmax(Q K^T / sqrt(D)) V; dV = P^T dO; dP = dO V^T;
 *     dS = P (dP - rowsum(O dO)) / sqrt(D); dQ = dS K; dK = dS^T Q; plus an
 *     optional causal mask (key j visible to query i iff j <= i), which the
 *     reference does not have.
 *
 *  2. oracle_reference_{forward,backward}_emul: float64 emulation of the
 *     reference's own kernels, step by step and with their 32x32 tiling
 *     (flash_attention.cu:57-169 and :226-326), including two behaviours of
 *     the reference that the exact path does not share:
 *       - keys past T are zero vectors that still enter the row max and the
 *         denominator (flash_attention.cu:104-109, :126-141);
 *       - the backward adds sum_k dS[y][k] * Q[y] into key row tile+y and
 *         sum_k P[y][k] * dO[y] into value row tile+y (:310-321), i.e. it
 *         uses the query row index y as the key row index.
 *     It is pinned against the reference's CUDA kernels on a B200 (tests
 *     that load oracle/_ref) and documents the divergence.
 *
 *  3. oracle_cpu_attention_fwd_bwd_f32: fp32 forward + backward with OpenMP
 *     over heads -- the CPU attention baseline timed by bench.py.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int visible(long i, long j, int causal) { return !causal || j <= i; }

/* ------------------------------------------------------------------------ */
/* 1. exact fp64                                                             */
/* ------------------------------------------------------------------------ */
void oracle_attention_forward_f64(const double* q, const double* k, const double* v, double* o, double* lse,
                                  long BH, long T, long D, int causal) {
  const double scale = 1.0 / sqrt((double)D);
#pragma omp parallel for schedule(dynamic) if (BH * T * T * D > 100000000L)
  for (long bh = 0; bh < BH; ++bh) {
    double* srow = (double*)malloc(sizeof(double) * (size_t)T);
    const double* Q = q + bh * T * D;
    const double* K = k + bh * T * D;
    const double* V = v + bh * T * D;
    for (long i = 0; i < T; ++i) {
      double m = -INFINITY;
      for (long j = 0; j < T; ++j) {
        if (!visible(i, j, causal)) continue;
        double acc = 0.0;
        for (long d = 0; d < D; ++d) acc += Q[i * D + d] * K[j * D + d];
        srow[j] = acc * scale;
        if (srow[j] > m) m = srow[j];
      }
      double l = 0.0;
      for (long j = 0; j < T; ++j) {
        if (!visible(i, j, causal)) continue;
        srow[j] = exp(srow[j] - m);
        l += srow[j];
      }
      double* O = o + (bh * T + i) * D;
      for (long d = 0; d < D; ++d) O[d] = 0.0;
      for (long j = 0; j < T; ++j) {
        if (!visible(i, j, causal)) continue;
        const double p = srow[j] / l;
        for (long d = 0; d < D; ++d) O[d] += p * V[j * D + d];
      }
      if (lse) lse[bh * T + i] = m + log(l);
    }
    free(srow);
  }
}

void oracle_attention_backward_f64(const double* q, const double* k, const double* v, const double* dO,
                                   double* dq, double* dk, double* dv, long BH, long T, long D, int causal) {
  const double scale = 1.0 / sqrt((double)D);
#pragma omp parallel for schedule(dynamic) if (BH * T * T * D > 100000000L)
  for (long bh = 0; bh < BH; ++bh) {
    const double* Q = q + bh * T * D;
    const double* K = k + bh * T * D;
    const double* V = v + bh * T * D;
    const double* G = dO + bh * T * D;
    double* dQ = dq + bh * T * D;
    double* dK = dk + bh * T * D;
    double* dV = dv + bh * T * D;
    double* P = (double*)malloc(sizeof(double) * (size_t)(T * T));
    double* O = (double*)calloc((size_t)(T * D), sizeof(double));
    memset(dQ, 0, sizeof(double) * T * D);
    memset(dK, 0, sizeof(double) * T * D);
    memset(dV, 0, sizeof(double) * T * D);
    for (long i = 0; i < T; ++i) {
      double m = -INFINITY;
      for (long j = 0; j < T; ++j) {
        double acc = 0.0;
        if (visible(i, j, causal)) {
          for (long d = 0; d < D; ++d) acc += Q[i * D + d] * K[j * D + d];
          acc *= scale;
          if (acc > m) m = acc;
        }
        P[i * T + j] = acc;
      }
      double l = 0.0;
      for (long j = 0; j < T; ++j) {
        const double e = visible(i, j, causal) ? exp(P[i * T + j] - m) : 0.0;
        P[i * T + j] = e;
        l += e;
      }
      for (long j = 0; j < T; ++j) {
        P[i * T + j] /= l;
        for (long d = 0; d < D; ++d) O[i * D + d] += P[i * T + j] * V[j * D + d];
      }
    }
    for (long i = 0; i < T; ++i) {
      double delta = 0.0;
      for (long d = 0; d < D; ++d) delta += O[i * D + d] * G[i * D + d];
      for (long j = 0; j < T; ++j) {
        const double p = P[i * T + j];
        if (p == 0.0) continue;
        double dp = 0.0;
        for (long d = 0; d < D; ++d) dp += G[i * D + d] * V[j * D + d];
        const double ds = p * (dp - delta) * scale;
        for (long d = 0; d < D; ++d) {
          dQ[i * D + d] += ds * K[j * D + d];
          dK[j * D + d] += ds * Q[i * D + d];
          dV[j * D + d] += p * G[i * D + d];
        }
      }
    }
    free(P);
    free(O);
  }
}

/* ------------------------------------------------------------------------ */
/* 2. emulation of the reference kernels (float64 arithmetic)               */
/* ------------------------------------------------------------------------ */
#define REF_TILE 32 /* BLOCKDIM, cuda_transformer/ModuleLayer.cu:6 */

void oracle_reference_forward_emul(const double* q, const double* k, const double* v, double* o,
                                   double* maxScores, double* denominators, long BH, long T, long D) {
  const double sq = sqrt((double)D);
  double sc[REF_TILE];
  for (long bh = 0; bh < BH; ++bh) {
    const double* Q = q + bh * T * D;
    const double* K = k + bh * T * D;
    const double* V = v + bh * T * D;
    for (long i = 0; i < T; ++i) {
      double maxScore = -1e20, den = 0.0;
      double* acc = o + (bh * T + i) * D; /* running weighted sum, normalised at the end */
      for (long d = 0; d < D; ++d) acc[d] = 0.0;
      for (long t0 = 0; t0 < T; t0 += REF_TILE) {
        double rowMax = -1e20;
        for (long x = 0; x < REF_TILE; ++x) {
          const long j = t0 + x;
          double s = 0.0;
          if (j < T)
            for (long d = 0; d < D; ++d) s += Q[i * D + d] * K[j * D + d];
          s /= sq; /* a padded key (zero vector) scores 0 */
          sc[x] = s;
          rowMax = fmax(rowMax, s);
        }
        const double newMax = fmax(maxScore, rowMax);
        const double rescale = exp(maxScore - newMax);
        double rowExpSum = 0.0;
        for (long x = 0; x < REF_TILE; ++x) {
          sc[x] = exp(sc[x] - newMax);
          rowExpSum += sc[x];
        }
        den = den * rescale + rowExpSum;
        for (long d = 0; d < D; ++d) {
          double w = 0.0;
          for (long x = 0; x < REF_TILE; ++x)
            if (t0 + x < T) w += sc[x] * V[(t0 + x) * D + d];
          acc[d] = acc[d] * rescale + w;
        }
        maxScore = newMax;
      }
      for (long d = 0; d < D; ++d) acc[d] /= den;
      if (maxScores) maxScores[bh * T + i] = maxScore;
      if (denominators) denominators[bh * T + i] = den;
    }
  }
}

/* Returns 0 on success, -1 when T is not a multiple of the 32-row tile (the
 * reference kernel then reads uninitialised shared memory for the rows past
 * T, so its result is undefined). */
int oracle_reference_backward_emul(const double* q, const double* k, const double* v, const double* o,
                                   const double* dO, const double* maxScores, const double* denominators,
                                   double* dq, double* dk, double* dv, long BH, long T, long D) {
  if (T % REF_TILE != 0) return -1;
  const double sq = sqrt((double)D);
  double P[REF_TILE * REF_TILE], dS[REF_TILE * REF_TILE];
  memset(dq, 0, sizeof(double) * BH * T * D);
  memset(dk, 0, sizeof(double) * BH * T * D);
  memset(dv, 0, sizeof(double) * BH * T * D);
  for (long bh = 0; bh < BH; ++bh) {
    const double* Q = q + bh * T * D;
    const double* K = k + bh * T * D;
    const double* V = v + bh * T * D;
    const double* O = o + bh * T * D;
    const double* G = dO + bh * T * D;
    double* dQ = dq + bh * T * D;
    double* dK = dk + bh * T * D;
    double* dV = dv + bh * T * D;
    for (long r0 = 0; r0 < T; r0 += REF_TILE) {    /* query tile (blockIdx.x) */
      for (long t0 = 0; t0 < T; t0 += REF_TILE) {  /* key tile (tileIdx) */
        for (long y = 0; y < REF_TILE; ++y) {      /* threadIdx.y */
          const long i = r0 + y;
          double delta = 0.0;
          for (long d = 0; d < D; ++d) delta += O[i * D + d] * G[i * D + d];
          for (long x = 0; x < REF_TILE; ++x) {    /* threadIdx.x */
            const long j = t0 + x;
            double s = 0.0, dp = 0.0;
            for (long d = 0; d < D; ++d) {
              s += Q[i * D + d] * K[j * D + d];
              dp += G[i * D + d] * V[j * D + d];
            }
            s /= sq;
            const double p = exp(s - maxScores[bh * T + i]) / denominators[bh * T + i];
            P[y * REF_TILE + x] = p;
            dS[y * REF_TILE + x] = p * (dp - delta) / sq;
          }
        }
        for (long y = 0; y < REF_TILE; ++y) {
          const long i = r0 + y;
          double sumDS = 0.0, sumP = 0.0;
          for (long x = 0; x < REF_TILE; ++x) {
            sumDS += dS[y * REF_TILE + x];
            sumP += P[y * REF_TILE + x];
          }
          for (long d = 0; d < D; ++d) {
            double dqv = 0.0;
            for (long x = 0; x < REF_TILE; ++x) dqv += dS[y * REF_TILE + x] * K[(t0 + x) * D + d];
            dQ[i * D + d] += dqv;
            /* key/value row t0 + y receives query row r0 + y's terms */
            dK[(t0 + y) * D + d] += sumDS * Q[i * D + d];
            dV[(t0 + y) * D + d] += sumP * G[i * D + d];
          }
        }
      }
    }
  }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* 3. CPU baseline: fp32 forward + backward, OpenMP over (batch, head)      */
/* ------------------------------------------------------------------------ */
void oracle_cpu_attention_fwd_bwd_f32(const float* q, const float* k, const float* v, const float* dO, float* o,
                                      float* lse, float* dq, float* dk, float* dv, long BH, long T, long D,
                                      int causal, int nthreads) {
  const float scale = 1.0f / sqrtf((float)D);
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#endif
#pragma omp parallel
  {
    float* P = (float*)malloc(sizeof(float) * (size_t)(T * T));
    float* dS = (float*)malloc(sizeof(float) * (size_t)T);
#pragma omp for schedule(dynamic)
    for (long bh = 0; bh < BH; ++bh) {
      const float* Q = q + bh * T * D;
      const float* K = k + bh * T * D;
      const float* V = v + bh * T * D;
      const float* G = dO + bh * T * D;
      float* O = o + bh * T * D;
      float* dQ = dq + bh * T * D;
      float* dK = dk + bh * T * D;
      float* dV = dv + bh * T * D;
      memset(dK, 0, sizeof(float) * T * D);
      memset(dV, 0, sizeof(float) * T * D);
      for (long i = 0; i < T; ++i) {
        const long jn = causal ? i + 1 : T;
        float m = -INFINITY;
        float* Pi = P + i * T;
        for (long j = 0; j < jn; ++j) {
          float acc = 0.f;
#pragma omp simd reduction(+ : acc)
          for (long d = 0; d < D; ++d) acc += Q[i * D + d] * K[j * D + d];
          Pi[j] = acc * scale;
          m = Pi[j] > m ? Pi[j] : m;
        }
        float l = 0.f;
        for (long j = 0; j < jn; ++j) {
          Pi[j] = expf(Pi[j] - m);
          l += Pi[j];
        }
        const float inv = 1.f / l;
        float* Oi = O + i * D;
        for (long d = 0; d < D; ++d) Oi[d] = 0.f;
        for (long j = 0; j < jn; ++j) {
          Pi[j] *= inv;
          const float p = Pi[j];
#pragma omp simd
          for (long d = 0; d < D; ++d) Oi[d] += p * V[j * D + d];
        }
        lse[bh * T + i] = m + logf(l);
      }
      for (long i = 0; i < T; ++i) {
        const long jn = causal ? i + 1 : T;
        const float* Pi = P + i * T;
        const float* Gi = G + i * D;
        float delta = 0.f;
#pragma omp simd reduction(+ : delta)
        for (long d = 0; d < D; ++d) delta += O[i * D + d] * Gi[d];
        for (long j = 0; j < jn; ++j) {
          float dp = 0.f;
#pragma omp simd reduction(+ : dp)
          for (long d = 0; d < D; ++d) dp += Gi[d] * V[j * D + d];
          dS[j] = Pi[j] * (dp - delta) * scale;
        }
        float* dQi = dQ + i * D;
        for (long d = 0; d < D; ++d) dQi[d] = 0.f;
        for (long j = 0; j < jn; ++j) {
          const float s = dS[j], p = Pi[j];
#pragma omp simd
          for (long d = 0; d < D; ++d) {
            dQi[d] += s * K[j * D + d];
            dK[j * D + d] += s * Q[i * D + d];
            dV[j * D + d] += p * Gi[d];
          }
        }
      }
    }
    free(P);
    free(dS);
  }
}
