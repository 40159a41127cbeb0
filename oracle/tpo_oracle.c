/*
 * CPU oracle for the chamfer / knn all-pairs nearest-neighbour path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product links, loads or calls this
 * file: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg do,
 * and only as the checker (or the timed CPU baseline), never as the thing being
 * measured or shipped.
 *
 * It restates, in plain C, the arithmetic of the reference implementation
 * (satyajitghana/torch-point-ops v0.1.0; paths relative to that project):
 *
 *   nn_*        chamfer_dist_kernel, torch_point_ops/chamfer/csrc/cuda/chamfer.cu:37-167
 *               (one direction: per-query min + argmin, strict '<' inside a
 *               tile (:69) and strict '>' across tiles (:159) => lowest index
 *               wins ties; distance (b-a)x^2 + (b-a)y^2 + (b-a)z^2 (:64-67)).
 *   chamfer_bwd chamfer_dist_grad_kernel, chamfer.cu:200-234 (g = 2*grad,
 *               grad_a += g*(a-b), grad_b -= g*(a-b); direction 1 then 2,
 *               :254-263), accumulated here sequentially.
 *   knn_fwd     knn_cpu_forward, torch_point_ops/knn/csrc/knn.cpp:30-101
 *               (priority_queue of (dist, idx): keeps the K smallest by
 *               (dist, idx), output ascending; pad idx -1 / dist 0 (:44-45);
 *               dist accumulated as ((0 + t_x) + t_y) + t_z (:64-72)).
 *   knn_bwd     knn_cpu_backward, knn.cpp:104-164 (rows < lengths1,
 *               k < min(K, lengths2), skip idx -1; L2: 2*g*(p1-p2); L1: g*sign)
 *               with the L1 sign at equality taken from the CUDA kernel
 *               (knn.cu:447-449: 0 when p1 == p2) when l1_zero_at_tie != 0.
 *
 *   fps         furthest_point_sampling_kernel, torch_point_ops/fps/csrc/cuda/fps.cu:108-213
 *               with its launch at :215-316 (the CUDA semantics, not the CPU
 *               path of fps/csrc/fps.cpp:17-88, which differs: it masks selected
 *               points and lets degenerate points win).  idx[0] = 0; temp starts
 *               at 1e10 (1e4 for fp16, :291); a point with |p|^2 <= 1e-3 is never
 *               updated nor chosen (:139-140); d = |p - p_old|^2 with the fma
 *               contraction below (:142), temp = min(d, temp) (:143); the argmax
 *               ties resolve as the reference's block reduction does: thread
 *               t = k mod bs keeps its first maximum in k order (strict '>',
 *               :145-146), and the halving tree (:152-205, __update :99-106)
 *               merges slot i with i+s for s = bs/2 .. 1 keeping slot i on ties,
 *               so bit 0 of the winning thread is decided last: among equal
 *               maxima the point with the smallest (bitreverse(k mod bs), k)
 *               wins, bs = min(512, 2^floor(log2 P)) (opt_n_threads,
 *               fps.cu:56-59).  If no point is valid the answer is 0 (besti's
 *               initial value, :131).
 *   gather_points gather_points_kernel / _grad_kernel, fps.cu:63-97
 *               (out[n,c,j] = points[n,c,idx[n,j]]; backward scatter-adds).
 *
 * Rounding modes (`mode`):
 *   0  "exact": every product and sum rounded separately, no contraction.
 *      This is the reference CPU path (g++ -O3 on x86-64 baseline emits no FMA).
 *   1  "fma":  t = dy*dy; t = fma(dx,dx,t); t = fma(dz,dz,t) -- the contraction
 *      nvcc applies to the reference CUDA chamfer kernel's x2*x2+y2*y2+z2*z2
 *      (chamfer.cu:67; default --fmad=true, setup.py:83-92 does not override it).
 *      Determined by comparing the reference CUDA build's outputs on a B200 with
 *      candidate orders (it matches this one bit for bit) and pinned by
 *      tests/test_ref_cuda_pin.py.  The reference CUDA knn kernels are NOT
 *      contracted (their outputs equal mode 0), so knn always uses mode 0.
 * fp16 follows c10::Half: every sub/mul/add rounds to half (round-to-nearest-
 * even), no fused operations, in both modes.
 *
 * Compile with -ffp-contract=off so that mode 0 really is uncontracted.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>

typedef _Float16 h16;

/* ---------------- distance kernels ---------------- */
static inline float d2_f32(int mode, float dx, float dy, float dz) {
  if (mode == 1) return fmaf(dz, dz, fmaf(dx, dx, dy * dy));
  float t = dx * dx;
  t = t + dy * dy;
  return t + dz * dz;
}
static inline double d2_f64(int mode, double dx, double dy, double dz) {
  if (mode == 1) return fma(dz, dz, fma(dx, dx, dy * dy));
  double t = dx * dx;
  t = t + dy * dy;
  return t + dz * dz;
}
static inline h16 hr(float v) { return (h16)v; }
static inline h16 d2_f16(h16 dx, h16 dy, h16 dz) {
  h16 sx = hr((float)dx * (float)dx);
  h16 sy = hr((float)dy * (float)dy);
  h16 sz = hr((float)dz * (float)dz);
  return hr((float)hr((float)sx + (float)sy) + (float)sz);
}

/* ------------- one direction of chamfer: min/argmin over the other cloud ------------- */
/* dist/idx for every query point of `a` (B,N,3) against `b` (B,M,3).  M == 0 leaves
 * zeros, as the reference's torch::zeros outputs (chamfer.cu:176-181). */
#define NN_BODY(T, D2)                                                          \
  _Pragma("omp parallel for collapse(2) schedule(static)")                     \
  for (int64_t bi = 0; bi < B; ++bi)                                           \
    for (int64_t i = 0; i < N; ++i) {                                          \
      const T* pa = a + (bi * N + i) * 3;                                      \
      const T* pb = b + bi * M * 3;                                            \
      T best = 0; int32_t bidx = 0;                                            \
      for (int64_t j = 0; j < M; ++j) {                                        \
        T dd = D2;                                                             \
        if (j == 0 || dd < best) { best = dd; bidx = (int32_t)j; }             \
      }                                                                        \
      dist[bi * N + i] = best; idx[bi * N + i] = bidx;                         \
    }

void oracle_nn_f32(int mode, int64_t B, int64_t N, int64_t M, const float* a,
                   const float* b, float* dist, int32_t* idx) {
  NN_BODY(float, d2_f32(mode, pb[j * 3] - pa[0], pb[j * 3 + 1] - pa[1], pb[j * 3 + 2] - pa[2]))
}
void oracle_nn_f64(int mode, int64_t B, int64_t N, int64_t M, const double* a,
                   const double* b, double* dist, int32_t* idx) {
  NN_BODY(double, d2_f64(mode, pb[j * 3] - pa[0], pb[j * 3 + 1] - pa[1], pb[j * 3 + 2] - pa[2]))
}
void oracle_nn_f16(int mode, int64_t B, int64_t N, int64_t M, const h16* a,
                   const h16* b, h16* dist, int32_t* idx) {
  (void)mode;
  NN_BODY(h16, d2_f16(hr((float)pb[j * 3] - (float)pa[0]),
                      hr((float)pb[j * 3 + 1] - (float)pa[1]),
                      hr((float)pb[j * 3 + 2] - (float)pa[2])))
}

/* ------------- chamfer backward (sequential accumulation) ------------- */
#define CBWD_DIR(T, MUL2, SUBV, ACC)                                           \
  for (int64_t bi = 0; bi < B; ++bi)                                           \
    for (int64_t i = 0; i < n; ++i) {                                          \
      const T* pa = a + (bi * n + i) * 3;                                      \
      int64_t j = idx[bi * n + i];                                             \
      const T* pb = b + (bi * m + j) * 3;                                      \
      T g = MUL2(gd[bi * n + i]);                                              \
      for (int d = 0; d < 3; ++d) {                                            \
        T v = SUBV(g, pa[d], pb[d]);                                           \
        ACC(ga[(bi * n + i) * 3 + d], v);                                      \
        ACC(gb[(bi * m + j) * 3 + d], -v);                                     \
      }                                                                        \
    }

#define MUL2_F(x) ((x) * 2)
#define SUBV_F(g, x, y) ((g) * ((x) - (y)))
#define ACC_F(dst, v) ((dst) += (v))
#define MUL2_H(x) hr((float)(x) * 2.0f)
#define SUBV_H(g, x, y) hr((float)(g) * (float)hr((float)(x) - (float)(y)))
#define ACC_H(dst, v) ((dst) = hr((float)(dst) + (float)(v)))

static void cbwd_f32(int64_t B, int64_t n, int64_t m, const float* a, const float* b,
                     const float* gd, const int32_t* idx, float* ga, float* gb) {
  CBWD_DIR(float, MUL2_F, SUBV_F, ACC_F)
}
static void cbwd_f64(int64_t B, int64_t n, int64_t m, const double* a, const double* b,
                     const double* gd, const int32_t* idx, double* ga, double* gb) {
  CBWD_DIR(double, MUL2_F, SUBV_F, ACC_F)
}
static void cbwd_f16(int64_t B, int64_t n, int64_t m, const h16* a, const h16* b,
                     const h16* gd, const int32_t* idx, h16* ga, h16* gb) {
  CBWD_DIR(h16, MUL2_H, SUBV_H, ACC_H)
}

/* grad1 (B,N,3) and grad2 (B,M,3) must be zeroed by the caller. */
void oracle_chamfer_bwd_f32(int64_t B, int64_t N, int64_t M, const float* x1, const float* x2,
                            const int32_t* i1, const int32_t* i2, const float* g1,
                            const float* g2, float* gx1, float* gx2) {
  if (M > 0) cbwd_f32(B, N, M, x1, x2, g1, i1, gx1, gx2);
  if (N > 0) cbwd_f32(B, M, N, x2, x1, g2, i2, gx2, gx1);
}
void oracle_chamfer_bwd_f64(int64_t B, int64_t N, int64_t M, const double* x1, const double* x2,
                            const int32_t* i1, const int32_t* i2, const double* g1,
                            const double* g2, double* gx1, double* gx2) {
  if (M > 0) cbwd_f64(B, N, M, x1, x2, g1, i1, gx1, gx2);
  if (N > 0) cbwd_f64(B, M, N, x2, x1, g2, i2, gx2, gx1);
}
void oracle_chamfer_bwd_f16(int64_t B, int64_t N, int64_t M, const h16* x1, const h16* x2,
                            const int32_t* i1, const int32_t* i2, const h16* g1,
                            const h16* g2, h16* gx1, h16* gx2) {
  if (M > 0) cbwd_f16(B, N, M, x1, x2, g1, i1, gx1, gx2);
  if (N > 0) cbwd_f16(B, M, N, x2, x1, g2, i2, gx2, gx1);
}

/* ------------- knn forward: K smallest by (dist, idx), ascending ------------- */
/* Keeps a sorted array of at most K entries.  A candidate is taken when fewer
 * than K are held or when it is strictly below the current worst (knn.cpp:74-80);
 * since candidates arrive in increasing index, an equal distance never displaces
 * an earlier index, and the insertion point after all entries with dist <= d
 * keeps the (dist, idx) order of the reference's priority_queue pop sequence. */
#define KNN_BODY(T, DIST_L2, DIST_L1)                                          \
  _Pragma("omp parallel for collapse(2) schedule(dynamic, 16)")                \
  for (int64_t n = 0; n < Nb; ++n)                                             \
    for (int64_t i = 0; i < P1; ++i) {                                         \
      T* od = dists + (n * P1 + i) * K;                                        \
      int64_t* oi = idxs + (n * P1 + i) * K;                                   \
      for (int64_t k = 0; k < K; ++k) { od[k] = (T)0; oi[k] = -1; }            \
      if (i >= len1[n]) continue;                                              \
      const T* pa = p1 + (n * P1 + i) * D;                                     \
      const T* pbase = p2 + n * P2 * D;                                        \
      int64_t cnt = 0;                                                         \
      for (int64_t j = 0; j < len2[n]; ++j) {                                  \
        const T* pb = pbase + j * D;                                           \
        T dd = (norm == 1) ? DIST_L1 : DIST_L2;                                \
        if (cnt < K || dd < od[cnt - 1]) {                                     \
          int64_t pos = (cnt < K) ? cnt : K - 1;                               \
          while (pos > 0 && od[pos - 1] > dd) {                                \
            od[pos] = od[pos - 1]; oi[pos] = oi[pos - 1]; --pos;               \
          }                                                                    \
          od[pos] = dd; oi[pos] = j;                                           \
          if (cnt < K) ++cnt;                                                  \
        }                                                                      \
      }                                                                        \
    }

static inline float l2_f32(int mode, int64_t D, const float* x, const float* y) {
  if (D == 3) return d2_f32(mode, x[0] - y[0], x[1] - y[1], x[2] - y[2]);
  float t = 0;
  for (int64_t d = 0; d < D; ++d) {
    float df = x[d] - y[d];
    t = (mode == 1) ? fmaf(df, df, t) : t + df * df;
  }
  return t;
}
static inline double l2_f64(int mode, int64_t D, const double* x, const double* y) {
  if (D == 3) return d2_f64(mode, x[0] - y[0], x[1] - y[1], x[2] - y[2]);
  double t = 0;
  for (int64_t d = 0; d < D; ++d) {
    double df = x[d] - y[d];
    t = (mode == 1) ? fma(df, df, t) : t + df * df;
  }
  return t;
}
static inline h16 l2_f16(int64_t D, const h16* x, const h16* y) {
  h16 t = 0;
  for (int64_t d = 0; d < D; ++d) {
    h16 df = hr((float)x[d] - (float)y[d]);
    t = hr((float)t + (float)hr((float)df * (float)df));
  }
  return t;
}
static inline float l1_f32(int64_t D, const float* x, const float* y) {
  float t = 0;
  for (int64_t d = 0; d < D; ++d) t = t + fabsf(x[d] - y[d]);
  return t;
}
static inline double l1_f64(int64_t D, const double* x, const double* y) {
  double t = 0;
  for (int64_t d = 0; d < D; ++d) t = t + fabs(x[d] - y[d]);
  return t;
}
static inline h16 l1_f16(int64_t D, const h16* x, const h16* y) {
  h16 t = 0;
  for (int64_t d = 0; d < D; ++d) {
    float df = (float)hr((float)x[d] - (float)y[d]);
    t = hr((float)t + fabsf(df));
  }
  return t;
}

void oracle_knn_f32(int mode, int64_t Nb, int64_t P1, int64_t P2, int64_t D, const float* p1,
                    const float* p2, const int64_t* len1, const int64_t* len2, int64_t norm,
                    int64_t K, float* dists, int64_t* idxs) {
  KNN_BODY(float, l2_f32(mode, D, pa, pb), l1_f32(D, pa, pb))
}
void oracle_knn_f64(int mode, int64_t Nb, int64_t P1, int64_t P2, int64_t D, const double* p1,
                    const double* p2, const int64_t* len1, const int64_t* len2, int64_t norm,
                    int64_t K, double* dists, int64_t* idxs) {
  KNN_BODY(double, l2_f64(mode, D, pa, pb), l1_f64(D, pa, pb))
}
void oracle_knn_f16(int mode, int64_t Nb, int64_t P1, int64_t P2, int64_t D, const h16* p1,
                    const h16* p2, const int64_t* len1, const int64_t* len2, int64_t norm,
                    int64_t K, h16* dists, int64_t* idxs) {
  (void)mode;
  KNN_BODY(h16, l2_f16(D, pa, pb), l1_f16(D, pa, pb))
}

/* ------------- knn backward (sequential accumulation) ------------- */
#define KBWD_BODY(T, L2V, L1V, ACC)                                            \
  for (int64_t n = 0; n < Nb; ++n) {                                           \
    int64_t kk = len2[n] < K ? len2[n] : K;                                    \
    for (int64_t i = 0; i < len1[n]; ++i)                                      \
      for (int64_t k = 0; k < kk; ++k) {                                       \
        int64_t j = idxs[(n * P1 + i) * K + k];                                \
        if (j == -1) continue;                                                 \
        T g = gd[(n * P1 + i) * K + k];                                        \
        for (int64_t d = 0; d < D; ++d) {                                      \
          T x = p1[(n * P1 + i) * D + d], y = p2[(n * P2 + j) * D + d];        \
          T v = (norm == 1) ? L1V : L2V;                                       \
          ACC(g1[(n * P1 + i) * D + d], v);                                    \
          ACC(g2[(n * P2 + j) * D + d], -v);                                   \
        }                                                                      \
      }                                                                        \
  }
#define SIGNV(T, x, y, g) ((x) > (y) ? (g) : ((l1_zero_at_tie && (x) == (y)) ? (T)0 : -(g)))

void oracle_knn_bwd_f32(int64_t Nb, int64_t P1, int64_t P2, int64_t D, const float* p1,
                        const float* p2, const int64_t* len1, const int64_t* len2,
                        const int64_t* idxs, int64_t norm, int64_t K, const float* gd,
                        int l1_zero_at_tie, float* g1, float* g2) {
  KBWD_BODY(float, (g * 2) * (x - y), SIGNV(float, x, y, g), ACC_F)
}
void oracle_knn_bwd_f64(int64_t Nb, int64_t P1, int64_t P2, int64_t D, const double* p1,
                        const double* p2, const int64_t* len1, const int64_t* len2,
                        const int64_t* idxs, int64_t norm, int64_t K, const double* gd,
                        int l1_zero_at_tie, double* g1, double* g2) {
  KBWD_BODY(double, (g * 2) * (x - y), SIGNV(double, x, y, g), ACC_F)
}
void oracle_knn_bwd_f16(int64_t Nb, int64_t P1, int64_t P2, int64_t D, const h16* p1,
                        const h16* p2, const int64_t* len1, const int64_t* len2,
                        const int64_t* idxs, int64_t norm, int64_t K, const h16* gd,
                        int l1_zero_at_tie, h16* g1, h16* g2) {
  KBWD_BODY(h16, hr((float)hr((float)g * 2.0f) * (float)hr((float)x - (float)y)),
            SIGNV(h16, x, y, g), ACC_H)
}

/* ---------------- furthest point sampling (reference CUDA semantics) ---------------- */
static int64_t fps_block_size(int64_t P) {
  int64_t bs = 1;
  while (bs * 2 <= P && bs < 512) bs *= 2;
  return bs;
}
static int64_t bitrev(int64_t c, int64_t bs) {
  int64_t r = 0;
  for (int64_t b = 1; b < bs; b <<= 1) r = (r << 1) | ((c & b) ? 1 : 0);
  return r;
}
/* Visit order of the reference's tie resolution: (bitreverse(k mod bs), k). */
#define FPS_BODY(T, LARGE, MAG, DIST, VALID)                                   \
  const int64_t bs = fps_block_size(P);                                        \
  T* temp = (T*)malloc(sizeof(T) * (P > 0 ? P : 1));                           \
  for (int64_t b = 0; b < B; ++b) {                                            \
    const T* pts = points + b * P * 3;                                         \
    int64_t* out = idx + b * S;                                                \
    if (S <= 0) continue;                                                      \
    for (int64_t k = 0; k < P; ++k) temp[k] = (T)(LARGE);                      \
    int64_t old = 0;                                                           \
    out[0] = 0;                                                                \
    for (int64_t j = 1; j < S; ++j) {                                          \
      const T x1 = pts[old * 3], y1 = pts[old * 3 + 1], z1 = pts[old * 3 + 2]; \
      T best = (T)(-1.0f);                                                     \
      int64_t besti = 0;                                                       \
      int have = 0;                                                            \
      for (int64_t c = 0; c < bs; ++c)                                         \
        for (int64_t k = bitrev(c, bs); k < P; k += bs) {                      \
          const T x2 = pts[k * 3], y2 = pts[k * 3 + 1], z2 = pts[k * 3 + 2];   \
          const T mag = MAG;                                                   \
          if (!(VALID)) continue;                                              \
          const T d = DIST;                                                    \
          const T d2 = (d < temp[k]) ? d : temp[k];                            \
          temp[k] = d2;                                                        \
          if (!have || d2 > best) { best = d2; besti = k; have = 1; }          \
        }                                                                      \
      old = have ? besti : 0;                                                  \
      out[j] = old;                                                            \
    }                                                                          \
  }                                                                            \
  free(temp);

void oracle_fps_f32(int64_t B, int64_t P, int64_t S, const float* points, int64_t* idx) {
  FPS_BODY(float, 1e10f, fmaf(z2, z2, fmaf(x2, x2, y2 * y2)),
           d2_f32(1, x2 - x1, y2 - y1, z2 - z1), mag > 1e-3f)
}
void oracle_fps_f64(int64_t B, int64_t P, int64_t S, const double* points, int64_t* idx) {
  FPS_BODY(double, 1e10, fma(z2, z2, fma(x2, x2, y2 * y2)),
           d2_f64(1, x2 - x1, y2 - y1, z2 - z1), mag > 1e-3)
}
void oracle_fps_f16(int64_t B, int64_t P, int64_t S, const h16* points, int64_t* idx) {
  const float thr = (float)(h16)1e-3f;
  FPS_BODY(h16, 1e4f,
           hr((float)hr((float)hr((float)x2 * (float)x2) + (float)hr((float)y2 * (float)y2)) +
              (float)hr((float)z2 * (float)z2)),
           d2_f16(hr((float)x2 - (float)x1), hr((float)y2 - (float)y1), hr((float)z2 - (float)z1)),
           (float)mag > thr)
}

/* gather_points: out (B,C,S) = points (B,C,P) at idx (B,S); backward scatter-add. */
#define GP_FWD(T)                                                              \
  for (int64_t b = 0; b < B; ++b)                                              \
    for (int64_t c = 0; c < C; ++c)                                            \
      for (int64_t j = 0; j < S; ++j)                                          \
        out[(b * C + c) * S + j] = points[(b * C + c) * P + idx[b * S + j]];
#define GP_BWD(T, ADD)                                                         \
  memset(gp, 0, sizeof(T) * B * C * P);                                        \
  for (int64_t b = 0; b < B; ++b)                                              \
    for (int64_t c = 0; c < C; ++c)                                            \
      for (int64_t j = 0; j < S; ++j) {                                        \
        T* dst = gp + (b * C + c) * P + idx[b * S + j];                        \
        *dst = ADD(*dst, go[(b * C + c) * S + j]);                             \
      }
#define ADD_PLAIN(a, v) ((a) + (v))
#define ADD_HALF(a, v) hr((float)(a) + (float)(v))
void oracle_gather_points_f32(int64_t B, int64_t C, int64_t P, int64_t S, const float* points,
                              const int64_t* idx, float* out) { GP_FWD(float) }
void oracle_gather_points_f64(int64_t B, int64_t C, int64_t P, int64_t S, const double* points,
                              const int64_t* idx, double* out) { GP_FWD(double) }
void oracle_gather_points_f16(int64_t B, int64_t C, int64_t P, int64_t S, const h16* points,
                              const int64_t* idx, h16* out) { GP_FWD(h16) }
void oracle_gather_points_bwd_f32(int64_t B, int64_t C, int64_t P, int64_t S, const float* go,
                                  const int64_t* idx, float* gp) { GP_BWD(float, ADD_PLAIN) }
void oracle_gather_points_bwd_f64(int64_t B, int64_t C, int64_t P, int64_t S, const double* go,
                                  const int64_t* idx, double* gp) { GP_BWD(double, ADD_PLAIN) }
void oracle_gather_points_bwd_f16(int64_t B, int64_t C, int64_t P, int64_t S, const h16* go,
                                  const int64_t* idx, h16* gp) { GP_BWD(h16, ADD_HALF) }
