/* hxb_oracle.c -- CPU restatement of the reference's hot-path semantics.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker for the CUDA dispatch
 * library and the CPU baseline of bench.py; nothing in the product links,
 * loads or calls it.
 *
 * The reference's own implementation of these dispatches (IREE's llvm-cpu
 * lowering and the Hexagon HMX codegen) cannot be built in this environment:
 * the third-party/iree, llvm-project and hexagon-mlir submodules are empty
 * and there is no network. So this restates the linalg semantics the
 * reference compiles, operation by operation, with f32 arithmetic and the
 * f32 -> f16 truncation left to the caller (numpy's round-to-nearest-even,
 * the same as arith.truncf):
 *
 *   hxo_matmul_f16       examples/matmul/matmul.mlir:2-12 (fill 0 or an
 *                        init, linalg.matmul accumulating into it) and the
 *                        HMX unpack's add-into-destination
 *                        (plugins/runtime/hexagon/dsp/ukernel/hmx/hmx.c:334-336)
 *   hxo_matmul_w8a16     the linalg the W8 dispatch is built from: sitofp
 *                        i8->f32, extf scale->f32, mulf, f32 contraction
 *   hxo_attention        examples/attention_layer/attention_layer.mlir:17-111:
 *                        extf, Q*s and K^T*s with s = sqrt(scale) rounded to
 *                        f32 (:12,32-45), f32 batch_matmul, row max (:53-61),
 *                        subf, math.exp, row sum, divf (:63-84), rows whose
 *                        scores are all -inf select 0 (:86-103), f32 P.V
 *                        (:104-106)
 *
 * Every sum runs in increasing index order with separate multiply and add
 * roundings (built with -ffp-contract=off), as the scalar linalg loops do.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef _Float16 f16;

#define IB 32
#define JB 256

static inline int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

/* C[M,N] (f32) = init (or 0) + A[M,K] . B, B = [K,N] (tb = 0) or [N,K]. */
void hxo_matmul_f16(const f16 *A, int64_t lda, const f16 *B, int64_t ldb,
                    int tb, const float *init, int64_t ldi, float *C,
                    int64_t ldc, int64_t M, int64_t N, int64_t K) {
  const int64_t nib = (M + IB - 1) / IB, njb = (N + JB - 1) / JB;
#pragma omp parallel for schedule(dynamic) collapse(2)
  for (int64_t ib = 0; ib < nib; ++ib) {
    for (int64_t jb = 0; jb < njb; ++jb) {
      float acc[IB][JB];
      float brow[JB];
      const int64_t i0 = ib * IB, i1 = min64(M, i0 + IB);
      const int64_t j0 = jb * JB, j1 = min64(N, j0 + JB);
      const int64_t nj = j1 - j0;
      for (int64_t i = i0; i < i1; ++i)
        for (int64_t j = 0; j < nj; ++j)
          acc[i - i0][j] = init ? init[i * ldi + j0 + j] : 0.0f;
      for (int64_t k = 0; k < K; ++k) {
        for (int64_t j = 0; j < nj; ++j)
          brow[j] = tb ? (float)B[(j0 + j) * ldb + k] : (float)B[k * ldb + j0 + j];
        for (int64_t i = i0; i < i1; ++i) {
          const float a = (float)A[i * lda + k];
          float *r = acc[i - i0];
          for (int64_t j = 0; j < nj; ++j) r[j] = r[j] + a * brow[j];
        }
      }
      for (int64_t i = i0; i < i1; ++i)
        memcpy(C + i * ldc + j0, acc[i - i0], (size_t)nj * sizeof(float));
    }
  }
}

/* C[M,N] (f32) = sum_k f32(A[m,k]) * (f32(W[k,n]) * f32(scale[n])). */
void hxo_matmul_w8a16(const f16 *A, int64_t lda, const int8_t *W, int64_t ldw,
                      const f16 *scale, float *C, int64_t ldc, int64_t M,
                      int64_t N, int64_t K) {
  const int64_t nib = (M + IB - 1) / IB, njb = (N + JB - 1) / JB;
#pragma omp parallel for schedule(dynamic) collapse(2)
  for (int64_t ib = 0; ib < nib; ++ib) {
    for (int64_t jb = 0; jb < njb; ++jb) {
      float acc[IB][JB];
      float brow[JB], s[JB];
      const int64_t i0 = ib * IB, i1 = min64(M, i0 + IB);
      const int64_t j0 = jb * JB, j1 = min64(N, j0 + JB);
      const int64_t nj = j1 - j0;
      for (int64_t j = 0; j < nj; ++j) s[j] = (float)scale[j0 + j];
      for (int64_t i = i0; i < i1; ++i)
        for (int64_t j = 0; j < nj; ++j) acc[i - i0][j] = 0.0f;
      for (int64_t k = 0; k < K; ++k) {
        for (int64_t j = 0; j < nj; ++j)
          brow[j] = (float)W[k * ldw + j0 + j] * s[j];
        for (int64_t i = i0; i < i1; ++i) {
          const float a = (float)A[i * lda + k];
          float *r = acc[i - i0];
          for (int64_t j = 0; j < nj; ++j) r[j] = r[j] + a * brow[j];
        }
      }
      for (int64_t i = i0; i < i1; ++i)
        memcpy(C + i * ldc + j0, acc[i - i0], (size_t)nj * sizeof(float));
    }
  }
}

/* O[bh,i,:] (f32) = attention of one f16 [BH,Sq,D] x [BH,Skv,D] problem.
 * `s` is the per-operand scale the MLIR applies to Q and to K^T (the square
 * root of the softmax scale, already rounded to f32). causal masks key j when
 * j > i + (Skv - Sq). */
void hxo_attention(const f16 *Q, const f16 *Kt, const f16 *V, float *O,
                   int64_t BH, int64_t Sq, int64_t Skv, int64_t D, float s,
                   int causal) {
#pragma omp parallel for schedule(dynamic) collapse(2)
  for (int64_t bh = 0; bh < BH; ++bh) {
    for (int64_t i = 0; i < Sq; ++i) {
      float *S = (float *)malloc((size_t)Skv * sizeof(float));
      float q[512];
      const f16 *qr = Q + (bh * Sq + i) * D;
      for (int64_t d = 0; d < D; ++d) q[d] = (float)qr[d] * s;
      const int64_t lim = causal ? i + (Skv - Sq) : Skv - 1;
      float mx = -INFINITY;
      int all_neg_inf = 1;
      for (int64_t j = 0; j < Skv; ++j) {
        float acc = 0.0f;
        if (j > lim) {
          acc = -INFINITY;
        } else {
          const f16 *kr = Kt + (bh * Skv + j) * D;
          for (int64_t d = 0; d < D; ++d) acc = acc + q[d] * ((float)kr[d] * s);
        }
        S[j] = acc;
        if (acc > mx) mx = acc; /* arith.maximumf over the row */
        if (acc != -INFINITY) all_neg_inf = 0;
      }
      float sum = 0.0f;
      for (int64_t j = 0; j < Skv; ++j) {
        S[j] = expf(S[j] - mx);
        sum = sum + S[j];
      }
      float o[512];
      for (int64_t d = 0; d < D; ++d) o[d] = 0.0f;
      for (int64_t j = 0; j < Skv; ++j) {
        const float p = all_neg_inf ? 0.0f : S[j] / sum;
        const f16 *vr = V + (bh * Skv + j) * D;
        for (int64_t d = 0; d < D; ++d) o[d] = o[d] + p * (float)vr[d];
      }
      memcpy(O + (bh * Sq + i) * D, o, (size_t)D * sizeof(float));
      free(S);
    }
  }
}

/* Known-answer generator restated from the HMX simulator tests
 * (plugins/runtime/hexagon/dsp/ukernel/hmx/test/test_support.c:242-260 and
 * accumulator_test.c:14-31): a 32x32 activation of exactly representable
 * halves, a sparse weight (1 on the diagonal, 0.5 on the cyclic
 * super-diagonal) and the scalar product scaled by the number of
 * accumulations, rounded to f16. */
void hxo_hmx_known_answer(f16 *act, f16 *wt, f16 *out, uint32_t accumulations) {
  for (uint32_t r = 0; r < 32; ++r)
    for (uint32_t c = 0; c < 32; ++c) {
      act[r * 32 + c] = (f16)((int32_t)((r * 3u + c * 5u) % 9u) - 4) / (f16)2.0f;
      wt[r * 32 + c] = r == c ? (f16)1.0f : (c == (r + 1u) % 32u ? (f16)0.5f : (f16)0.0f);
    }
  for (uint32_t r = 0; r < 32; ++r)
    for (uint32_t c = 0; c < 32; ++c) {
      float v = 0.0f;
      for (uint32_t d = 0; d < 32; ++d) v += (float)act[r * 32 + d] * (float)wt[d * 32 + c];
      out[r * 32 + c] = (f16)(v * (float)accumulations);
    }
}
