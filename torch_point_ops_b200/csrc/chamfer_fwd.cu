// Chamfer forward: fused bidirectional nearest neighbour for sm_100a.
//
// Replaces the reference's chamfer_dist_kernel (torch_point_ops/chamfer/csrc/
// cuda/chamfer.cu:37-167), which runs the full (B,N,M) distance matrix twice,
// once per direction.  Here every (i,j) pair is evaluated ONCE and feeds both
// the row minimum (dist1/idx1) and the column minimum (dist2/idx2).
//
// Work decomposition.  A CTA takes a unit = (batch, row block, column segment).
// Each warp owns 32 lanes x R consecutive rows held in registers; the CTA's
// warps share the column segment, staged 256 columns at a time into shared
// memory (coordinates duplicated into {c,c} pairs so one packed fp32x2 op
// serves two rows).  A step processes 4 columns against the lane's R rows:
//   * row side   : running min per row (3-input FMNMX) + the 4-column chunk in
//                  which it last strictly improved (strict '<' in increasing
//                  column order => lowest column on ties);
//   * column side: min over the lane's R rows, then a warp-wide redux.min on
//                  the (non-negative float) bit pattern and a ballot for the
//                  lowest lane holding it (=> lowest row chunk on ties).
// Partial results are packed keys  (distance bits << 32) | chunk start  and
// merged across warps (shared memory) and CTAs (global atomic min).  Because the
// distance is >= 0 its bit pattern orders like the value, so the key order is
// (distance, index) -- exactly the reference's tie rule (chamfer.cu:69 strict
// '<' inside a tile, :159 strict '>' across tiles => lowest index wins).
// A finalize pass decodes each key and rescans its chunk (4 columns or R rows)
// with the identical arithmetic to recover the exact index.
//
// fp32 runs on packed fp32x2 instructions; fp16 computes the c10::Half
// per-operation-rounded distance and runs the same float machinery on its exact
// float value; fp64 uses 128-bit keys merged by a 16-byte compare-and-swap.
#include "tpo_internal.h"

namespace tpo {

// ----------------------------- fp32 fast path -----------------------------
// Set (kErrBulkTimeout) if a bounded wait for a bulk copy ever gave up; read by
// tpo_device_error_flags().
static __device__ unsigned g_fwd_device_error = 0;
#ifndef TPO_CF_R
#define TPO_CF_R 16
#endif
#ifndef TPO_CF_MINB
#define TPO_CF_MINB 1
#endif
#ifndef TPO_CF_SUNROLL
#define TPO_CF_SUNROLL 2
#endif
constexpr int CF_SUNROLL = TPO_CF_SUNROLL;
constexpr int CF_R = TPO_CF_R;        // rows per lane
constexpr int CF_RP = CF_R / 2;       // packed row pairs per lane
constexpr int CF_C = 4;               // columns per sub-step
#ifndef TPO_CF_HS
#define TPO_CF_HS 2
#endif
constexpr int CF_CHUNK = TPO_CF_HS * CF_C;  // fp32 row-side chunk (columns per key)
constexpr int CF_HS = CF_CHUNK / CF_C;  // sub-steps per chunk
constexpr int CH_CHUNK = 2 * CF_C;      // fp16 row-side chunk
constexpr int CF_TILE_STEPS = 64;     // steps per shared-memory tile
constexpr int CF_TILE = CF_TILE_STEPS * CF_C;
#ifndef TPO_CF_MAXW
#define TPO_CF_MAXW 4
#endif
constexpr int CF_MAXW = TPO_CF_MAXW;  // warps per CTA
constexpr int CF_ROWS_PER_WARP = 32 * CF_R;

// min over R values with 3-input FMNMX, as a balanced tree
template <int R>
__device__ __forceinline__ float col_min(const float* v) {
  if constexpr (R == 16) {
    const float m5 = min3f(min3f(v[0], v[1], v[2]), min3f(v[3], v[4], v[5]), min3f(v[6], v[7], v[8]));
    const float m6 = min3f(min3f(v[9], v[10], v[11]), min3f(v[12], v[13], v[14]), v[15]);
    return fminf(m5, m6);
  } else if constexpr (R == 8) {
    return min3f(min3f(v[0], v[1], v[2]), min3f(v[3], v[4], v[5]), fminf(v[6], v[7]));
  } else {
    float m = v[0];
    int i = 1;
#pragma unroll
    for (; i + 1 < R; i += 2) m = min3f(m, v[i], v[i + 1]);
    if (i < R) m = fminf(m, v[i]);
    return m;
  }
}

__device__ __forceinline__ void block_sum2(double& a, double& c, double* sa, double* sc) {
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    a += __shfl_down_sync(0xffffffffu, a, off);
    c += __shfl_down_sync(0xffffffffu, c, off);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) { sa[warp] = a; sc[warp] = c; }
  __syncthreads();
  a = 0.0;
  c = 0.0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) { a += sa[w]; c += sc[w]; }
}

__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

template <int MODE>
__global__ void __launch_bounds__(CF_MAXW * 32, TPO_CF_MINB)
    chamfer_keys_f32_kernel(const float* __restrict__ xyz1, const float* __restrict__ xyz2,
                            int64_t N, int64_t M, int64_t row_begin, int64_t row_end,
                            int rb_count, int cs_count, int64_t seg,
                            u64* __restrict__ keys1, u64* __restrict__ keys2) {
  __shared__ __align__(16) float2 s_col[CF_TILE_STEPS][3][CF_C];
  __shared__ __align__(16) uint2 s_wb[CF_MAXW][CF_TILE];  // {ballot, distance bits}

  pdl_wait();  // launched with programmatic serialisation: inputs/keys ready after this
  const int W = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int64_t unit = blockIdx.x;
  const int cs = (int)(unit % cs_count);
  unit /= cs_count;
  const int rb = (int)(unit % rb_count);
  const int64_t b = unit / rb_count;
  const int64_t c0 = (int64_t)cs * seg;
  const int64_t c1 = min(M, c0 + seg);
  const int64_t blk_row0 = row_begin + (int64_t)rb * W * CF_ROWS_PER_WARP;
  const int64_t warp_row0 = blk_row0 + (int64_t)warp * CF_ROWS_PER_WARP;
  const int64_t lane_row0 = warp_row0 + (int64_t)lane * CF_R;
  const bool warp_active = warp_row0 < row_end;
  const int n_active = (int)min64(W, (row_end - blk_row0 + CF_ROWS_PER_WARP - 1) / CF_ROWS_PER_WARP);
  const float qnan = __int_as_float(0x7fffffff);

  // The CTA's rows, staged once in shared memory (lanes read their R rows from
  // here; the column merge rescans winning row chunks here), and each column
  // tile, land by 1-D bulk copies (TMA) on one mbarrier; unaligned heads/tails
  // and NaN padding are filled by plain loads meanwhile.
  __shared__ __align__(16) float s_rows[CF_MAXW * CF_ROWS_PER_WARP * 3];
  __shared__ __align__(16) float s_raw[CF_TILE * 3];
  __shared__ __align__(8) unsigned long long s_bar;
  unsigned phase = 0;
  if (threadIdx.x == 0) mbar_init(&s_bar, 1);
  __syncthreads();
  const int64_t nrow = min64((int64_t)W * CF_ROWS_PER_WARP, max64(row_end - blk_row0, 0));
  auto stage = [&](bool with_rows, int64_t tc) {
    const float* rsrc = xyz1 + (b * N + blk_row0) * 3;
    const int rfl = with_rows ? (int)(nrow * 3) : 0;  // row floats to load
    const int rbulk = (((uintptr_t)rsrc & 15) == 0) ? (rfl & ~3) : 0;
    const int ncols = (int)min64(CF_TILE, c1 - tc);
    const float* tsrc = xyz2 + (b * M + tc) * 3;
    const int tfl = ncols * 3;
    const int tbulk = (((uintptr_t)tsrc & 15) == 0) ? (tfl & ~3) : 0;
    if (threadIdx.x == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_expect_tx(&s_bar, (unsigned)(rbulk + tbulk) * 4u);
      if (rbulk) bulk_g2s(s_rows, rsrc, (unsigned)rbulk * 4u, &s_bar);
      if (tbulk) bulk_g2s(s_raw, tsrc, (unsigned)tbulk * 4u, &s_bar);
    }
    if (with_rows)
      for (int e = rbulk + threadIdx.x; e < W * CF_ROWS_PER_WARP * 3; e += blockDim.x)
        s_rows[e] = e < rfl ? __ldg(rsrc + e) : qnan;
    for (int e = tbulk + threadIdx.x; e < tfl; e += blockDim.x) s_raw[e] = __ldg(tsrc + e);
    mbar_wait(&s_bar, phase, &g_fwd_device_error);
    phase ^= 1u;
    __syncthreads();
    // duplicated {c,c} layout, NaN-padded to whole chunks
    const int nsteps = ((ncols + CF_CHUNK - 1) / CF_CHUNK) * CF_HS;
    float2* dst = &s_col[0][0][0];
    for (int e = threadIdx.x; e < nsteps * CF_C * 3; e += blockDim.x) {
      const int col = e / 3;
      const int comp = e - col * 3;
      const float v = col < ncols ? s_raw[e] : qnan;
      dst[((col >> 2) * 3 + comp) * CF_C + (col & 3)] = make_float2(v, v);
    }
    __syncthreads();
  };
  if (c0 < c1) stage(true, c0);
  u64 QX[CF_RP], QY[CF_RP], QZ[CF_RP];
  {
    const float* a = s_rows + (warp * CF_ROWS_PER_WARP + lane * CF_R) * 3;
#pragma unroll
    for (int p = 0; p < CF_RP; ++p) {
      QX[p] = pk(a[6 * p + 0], a[6 * p + 3]);
      QY[p] = pk(a[6 * p + 1], a[6 * p + 4]);
      QZ[p] = pk(a[6 * p + 2], a[6 * p + 5]);
    }
  }
  float best[CF_R];
  int bchunk[CF_R];
#pragma unroll
  for (int r = 0; r < CF_R; ++r) {
    best[r] = __int_as_float(0x7f800000);
    bchunk[r] = 0;
  }

  for (int64_t tc = c0; tc < c1; tc += CF_TILE) {
    const int ncols = (int)min64(CF_TILE, c1 - tc);
    const int nsteps = ((ncols + CF_CHUNK - 1) / CF_CHUNK) * CF_HS;  // whole chunks
    if (tc != c0) {  // the first tile was staged together with the rows
      __syncthreads();
      stage(false, tc);
    }
    if (warp_active) {
      // Column side, software-pipelined: a sub-step folds its columns' minima
      // over the lane's rows (pend) and the warp-wide reduction of those is
      // issued during the next sub-step, off the dependency chain.
      unsigned pend[CF_C];
      int pend_slot = -1;
      // Two 4-column sub-steps per iteration; the row-side chunk is 8 columns.
#pragma unroll CF_SUNROLL
      for (int s = 0; s < nsteps; s += CF_HS) {
        float rm[CF_R];
#pragma unroll
        for (int h = 0; h < CF_HS; ++h) {
          if (pend_slot >= 0) {
#pragma unroll
            for (int c = 0; c < CF_C; ++c) {
              const unsigned w = redux_min_u32(pend[c]);
              const unsigned bal = __ballot_sync(0xffffffffu, pend[c] == w);
              if (lane == 0) s_wb[warp][pend_slot + c] = make_uint2(bal, w);
            }
          }
          const ulonglong2* cp = reinterpret_cast<const ulonglong2*>(&s_col[s + h][0][0]);
          const ulonglong2 xa = cp[0], xb = cp[1], ya = cp[2], yb = cp[3], za = cp[4], zb = cp[5];
          const u64 X[CF_C] = {xa.x, xa.y, xb.x, xb.y};
          const u64 Y[CF_C] = {ya.x, ya.y, yb.x, yb.y};
          const u64 Z[CF_C] = {za.x, za.y, zb.x, zb.y};
          float d[CF_C][CF_R];
#pragma unroll
          for (int c = 0; c < CF_C; ++c) {
#pragma unroll
            for (int p = 0; p < CF_RP; ++p) {
              const u64 t = dist2x2<MODE>(sub2(X[c], QX[p]), sub2(Y[c], QY[p]), sub2(Z[c], QZ[p]));
              upk(t, d[c][2 * p], d[c][2 * p + 1]);
            }
          }
#pragma unroll
          for (int r = 0; r < CF_R; ++r) {
            const float m = min3f(h == 0 ? best[r] : rm[r], d[0][r], d[1][r]);
            rm[r] = min3f(m, d[2][r], d[3][r]);
          }
          // column side: the lane's minimum over its rows per column; next
          // sub-step, the warp min of those (bit pattern of a non-negative float
          // orders like its value; NaN padding sorts last) and the ballot of
          // lanes holding it -- the winning lane's row is resolved at the merge
#pragma unroll
          for (int c = 0; c < CF_C; ++c) pend[c] = __float_as_uint(col_min<CF_R>(d[c]));
          pend_slot = (s + h) * CF_C;
        }
        const int colbase = (int)(tc + s * CF_C);
#pragma unroll
        for (int r = 0; r < CF_R; ++r) {
          if (rm[r] < best[r]) bchunk[r] = colbase;
          best[r] = rm[r];
        }
      }
      if (pend_slot >= 0) {  // the last sub-step's columns
#pragma unroll
        for (int c = 0; c < CF_C; ++c) {
          const unsigned w = redux_min_u32(pend[c]);
          const unsigned bal = __ballot_sync(0xffffffffu, pend[c] == w);
          if (lane == 0) s_wb[warp][pend_slot + c] = make_uint2(bal, w);
        }
      }
    }
    __syncthreads();
    // merge the warps' column results: the smallest distance, lowest warp (= lowest
    // rows) on ties; then rescan the winning lane's R rows in shared memory with
    // the identical arithmetic, so the key carries the exact lowest row index
    for (int col = threadIdx.x; col < ncols; col += blockDim.x) {
      unsigned bw = s_wb[0][col].y;
      int wb = 0;
      for (int w = 1; w < n_active; ++w) {
        const unsigned v = s_wb[w][col].y;
        if (v < bw) { bw = v; wb = w; }
      }
      const int lr0 = wb * CF_ROWS_PER_WARP + (__ffs(s_wb[wb][col].x) - 1) * CF_R;
      const float cx = s_col[col >> 2][0][col & 3].x;
      const float cy = s_col[col >> 2][1][col & 3].x;
      const float cz = s_col[col >> 2][2][col & 3].x;
      int found = 0;
#pragma unroll
      for (int k = CF_R - 1; k >= 0; --k) {
        const float* r = s_rows + (lr0 + k) * 3;
        const float dd = dist1f<MODE>(__fsub_rn(cx, r[0]), __fsub_rn(cy, r[1]), __fsub_rn(cz, r[2]));
        if (__float_as_uint(dd) == bw) found = k;
      }
      const u64 k = ((u64)bw << 32) | (unsigned)(blk_row0 + lr0 + found);
      red_min_u64(keys2 + b * M + tc + col, k);
    }
  }
  if (warp_active) {
#pragma unroll
    for (int r = 0; r < CF_R; ++r) {
      const int64_t row = lane_row0 + r;
      if (row < row_end)
        red_min_u64(keys1 + b * N + row,
                    ((u64)__float_as_uint(best[r]) << 32) | (unsigned)bchunk[r]);
    }
  }
  pdl_trigger();  // the next kernel may be scheduled (it waits for this grid)
}

// ----------------------------- fp16 fast path -----------------------------
// The fp32 kernel's structure on packed f16x2: a register holds the same
// coordinate of two rows, shared memory holds {c,c} per column, and every
// sub/mul/add rounds to half (c10::Half semantics, chamfer.cu:64-67).  Row minima
// are packed f16x2 mins; column minima reduce the half bit patterns (ordered
// like the values for d >= 0) with redux.sync.  Keys store the distance as the
// bits of its exact float value, like the generic path, so finalize is shared.
__device__ __forceinline__ unsigned short h_lo(h2 v) { return (unsigned short)(v & 0xffffu); }
__device__ __forceinline__ unsigned short h_hi(h2 v) { return (unsigned short)(v >> 16); }
__device__ __forceinline__ unsigned hbits_to_fbits(unsigned hb) {
  return __float_as_uint(__half2float(__ushort_as_half((unsigned short)hb)));
}

__global__ void __launch_bounds__(CF_MAXW * 32, TPO_CF_MINB)
    chamfer_keys_f16_kernel(const __half* __restrict__ xyz1, const __half* __restrict__ xyz2,
                            int64_t N, int64_t M, int64_t row_begin, int64_t row_end,
                            int rb_count, int cs_count, int64_t seg,
                            u64* __restrict__ keys1, u64* __restrict__ keys2) {
  __shared__ __align__(16) h2 s_col[CF_TILE_STEPS][3][CF_C];
  __shared__ __align__(16) uint2 s_wb[CF_MAXW][CF_TILE];  // {ballot, half distance bits}
  __shared__ __align__(16) __half s_rows[CF_MAXW * CF_ROWS_PER_WARP * 3];

  pdl_wait();  // launched with programmatic serialisation: inputs/keys ready after this
  const int W = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int64_t unit = blockIdx.x;
  const int cs = (int)(unit % cs_count);
  unit /= cs_count;
  const int rb = (int)(unit % rb_count);
  const int64_t b = unit / rb_count;
  const int64_t c0 = (int64_t)cs * seg;
  const int64_t c1 = min(M, c0 + seg);
  const int64_t blk_row0 = row_begin + (int64_t)rb * W * CF_ROWS_PER_WARP;
  const int64_t warp_row0 = blk_row0 + (int64_t)warp * CF_ROWS_PER_WARP;
  const int64_t lane_row0 = warp_row0 + (int64_t)lane * CF_R;
  const bool warp_active = warp_row0 < row_end;
  const int n_active = (int)min64(W, (row_end - blk_row0 + CF_ROWS_PER_WARP - 1) / CF_ROWS_PER_WARP);
  const unsigned short hnan = 0x7fff;

  // rows and column tiles by 1-D bulk copies on one mbarrier (as the fp32 kernel)
  __shared__ __align__(16) unsigned short s_raw[CF_TILE * 3];
  __shared__ __align__(8) unsigned long long s_bar;
  unsigned phase = 0;
  if (threadIdx.x == 0) mbar_init(&s_bar, 1);
  __syncthreads();
  const int64_t nrow = min64((int64_t)W * CF_ROWS_PER_WARP, max64(row_end - blk_row0, 0));
  unsigned short* s_rows16 = reinterpret_cast<unsigned short*>(s_rows);
  auto stage = [&](bool with_rows, int64_t tc) {
    const unsigned short* rsrc = reinterpret_cast<const unsigned short*>(xyz1 + (b * N + blk_row0) * 3);
    const int rfl = with_rows ? (int)(nrow * 3) : 0;
    const int rbulk = (((uintptr_t)rsrc & 15) == 0) ? (rfl & ~7) : 0;
    const int ncols = (int)min64(CF_TILE, c1 - tc);
    const unsigned short* tsrc = reinterpret_cast<const unsigned short*>(xyz2 + (b * M + tc) * 3);
    const int tfl = ncols * 3;
    const int tbulk = (((uintptr_t)tsrc & 15) == 0) ? (tfl & ~7) : 0;
    if (threadIdx.x == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_expect_tx(&s_bar, (unsigned)(rbulk + tbulk) * 2u);
      if (rbulk) bulk_g2s(s_rows16, rsrc, (unsigned)rbulk * 2u, &s_bar);
      if (tbulk) bulk_g2s(s_raw, tsrc, (unsigned)tbulk * 2u, &s_bar);
    }
    if (with_rows)
      for (int e = rbulk + threadIdx.x; e < W * CF_ROWS_PER_WARP * 3; e += blockDim.x)
        s_rows16[e] = e < rfl ? rsrc[e] : hnan;
    for (int e = tbulk + threadIdx.x; e < tfl; e += blockDim.x) s_raw[e] = tsrc[e];
    mbar_wait(&s_bar, phase, &g_fwd_device_error);
    phase ^= 1u;
    __syncthreads();
    const int nsteps = ((ncols + CH_CHUNK - 1) / CH_CHUNK) * 2;
    h2* dst = &s_col[0][0][0];
    for (int e = threadIdx.x; e < nsteps * CF_C * 3; e += blockDim.x) {
      const int col = e / 3;
      const int comp = e - col * 3;
      const unsigned short v = col < ncols ? s_raw[e] : hnan;
      dst[((col >> 2) * 3 + comp) * CF_C + (col & 3)] = hpk(v, v);
    }
    __syncthreads();
  };
  if (c0 < c1) stage(true, c0);
  h2 QX[CF_RP], QY[CF_RP], QZ[CF_RP];
  {
    const unsigned short* a = reinterpret_cast<const unsigned short*>(s_rows) +
                              (warp * CF_ROWS_PER_WARP + lane * CF_R) * 3;
#pragma unroll
    for (int p = 0; p < CF_RP; ++p) {
      QX[p] = hpk(a[6 * p + 0], a[6 * p + 3]);
      QY[p] = hpk(a[6 * p + 1], a[6 * p + 4]);
      QZ[p] = hpk(a[6 * p + 2], a[6 * p + 5]);
    }
  }
  h2 best[CF_RP];
  int bchunk[CF_R];
#pragma unroll
  for (int p = 0; p < CF_RP; ++p) best[p] = hpk(0x7c00, 0x7c00);  // +inf, +inf
#pragma unroll
  for (int r = 0; r < CF_R; ++r) bchunk[r] = 0;

  for (int64_t tc = c0; tc < c1; tc += CF_TILE) {
    const int ncols = (int)min64(CF_TILE, c1 - tc);
    const int nsteps = ((ncols + CH_CHUNK - 1) / CH_CHUNK) * 2;
    if (tc != c0) {
      __syncthreads();
      stage(false, tc);
    }
    if (warp_active) {
#pragma unroll 1
      for (int s = 0; s < nsteps; s += 2) {
        h2 rm[CF_RP];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint4 xa = *reinterpret_cast<const uint4*>(&s_col[s + h][0][0]);
          const uint4 ya = *reinterpret_cast<const uint4*>(&s_col[s + h][1][0]);
          const uint4 za = *reinterpret_cast<const uint4*>(&s_col[s + h][2][0]);
          const h2 X[CF_C] = {xa.x, xa.y, xa.z, xa.w};
          const h2 Y[CF_C] = {ya.x, ya.y, ya.z, ya.w};
          const h2 Z[CF_C] = {za.x, za.y, za.z, za.w};
          h2 d[CF_C][CF_RP];
#pragma unroll
          for (int c = 0; c < CF_C; ++c)
#pragma unroll
            for (int p = 0; p < CF_RP; ++p)
              d[c][p] = hdist2(hsub2r(X[c], QX[p]), hsub2r(Y[c], QY[p]), hsub2r(Z[c], QZ[p]));
#pragma unroll
          for (int p = 0; p < CF_RP; ++p) {
            const h2 m = hmin2r(h == 0 ? best[p] : rm[p], hmin2r(d[0][p], d[1][p]));
            rm[p] = hmin2r(m, hmin2r(d[2][p], d[3][p]));
          }
#pragma unroll
          for (int c = 0; c < CF_C; ++c) {
            h2 m = d[c][0];
#pragma unroll
            for (int p = 1; p < CF_RP; ++p) m = hmin2r(m, d[c][p]);
            const h2 mm = hmin2r(m, m >> 16);  // low half: min of both halves
            const unsigned u = mm & 0xffffu;
            const unsigned w = redux_min_u32(u);
            const unsigned bal = __ballot_sync(0xffffffffu, u == w);
            if (lane == 0) s_wb[warp][(s + h) * CF_C + c] = make_uint2(bal, w);
          }
        }
        const int colbase = (int)(tc + s * CF_C);
#pragma unroll
        for (int p = 0; p < CF_RP; ++p) {
          const unsigned lt = __hlt2_mask(*reinterpret_cast<const __half2*>(&rm[p]),
                                          *reinterpret_cast<const __half2*>(&best[p]));
          if (lt & 0xffffu) bchunk[2 * p] = colbase;
          if (lt >> 16) bchunk[2 * p + 1] = colbase;
          best[p] = rm[p];
        }
      }
    }
    __syncthreads();
    for (int col = threadIdx.x; col < ncols; col += blockDim.x) {
      unsigned bw = s_wb[0][col].y;
      int wb = 0;
      for (int w = 1; w < n_active; ++w) {
        const unsigned v = s_wb[w][col].y;
        if (v < bw) { bw = v; wb = w; }
      }
      const int lr0 = wb * CF_ROWS_PER_WARP + (__ffs(s_wb[wb][col].x) - 1) * CF_R;
      const __half cx = __ushort_as_half(h_lo(s_col[col >> 2][0][col & 3]));
      const __half cy = __ushort_as_half(h_lo(s_col[col >> 2][1][col & 3]));
      const __half cz = __ushort_as_half(h_lo(s_col[col >> 2][2][col & 3]));
      int found = 0;
#pragma unroll
      for (int k = CF_R - 1; k >= 0; --k) {
        const __half* r = s_rows + (lr0 + k) * 3;
        const __half dd = dist1h(hsub_rn(cx, r[0]), hsub_rn(cy, r[1]), hsub_rn(cz, r[2]));
        if ((unsigned)__half_as_ushort(dd) == bw) found = k;
      }
      const u64 k = ((u64)hbits_to_fbits(bw) << 32) | (unsigned)(blk_row0 + lr0 + found);
      red_min_u64(keys2 + b * M + tc + col, k);
    }
  }
  if (warp_active) {
#pragma unroll
    for (int p = 0; p < CF_RP; ++p) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = 2 * p + h;
        const int64_t row = lane_row0 + r;
        const unsigned hb = h ? h_hi(best[p]) : h_lo(best[p]);
        if (row < row_end)
          red_min_u64(keys1 + b * N + row, ((u64)hbits_to_fbits(hb) << 32) | (unsigned)bchunk[r]);
      }
    }
  }
  pdl_trigger();  // the next kernel may be scheduled (it waits for this grid)
}

// ------------------------- scalar distance helpers -------------------------
// Rescan widths of the fp64 keys in finalize: the keys carry exact indices, so
// a scan from the key's index finds it first.
constexpr int CG_R = 8;
constexpr int CG_C = 4;

template <typename T, int MODE>
struct GenDist;
template <int MODE>
struct GenDist<__half, MODE> {
  using V = float;  // exact float value of the half distance
  __device__ static float d(__half cx, __half cy, __half cz, __half qx, __half qy, __half qz) {
    return __half2float(dist1h(hsub_rn(cx, qx), hsub_rn(cy, qy), hsub_rn(cz, qz)));
  }
  __device__ static __half nan_() { return __ushort_as_half((unsigned short)0x7fff); }
};
template <int MODE>
struct GenDist<double, MODE> {
  using V = double;
  __device__ static double d(double cx, double cy, double cz, double qx, double qy, double qz) {
    return dist1d<MODE>(__dsub_rn(cx, qx), __dsub_rn(cy, qy), __dsub_rn(cz, qz));
  }
  __device__ static double nan_() { return __longlong_as_double(0x7fffffffffffffffll); }
};

// ----------------------------- fp64 fast path -----------------------------
// The fp32 kernel's structure for doubles, with the minima tracked on the
// distances' HIGH 32-bit words.  For d >= 0 the high word (sign, exponent, 20
// mantissa bits) is monotone in d, so integer minima of high words (3-input
// vimin3, on the integer pipe) keep the FP64 pipe for the distance itself
// (3 sub + 1 mul + 2 fma per pair).  The high word is only a proxy; exactness
// is restored before anything leaves the CTA:
//   * rows: the 4-column chunk where a row's high-word minimum was first reached
//     is rescanned in full precision at the end; if a later chunk reached the
//     SAME high word (a "tie", where a smaller low word could hide) the row's
//     whole column segment is rescanned instead;
//   * columns: every lane whose minimum high word equals the warp's minimum is
//     a candidate (the ballot), every warp whose minimum equals the CTA's is a
//     candidate, and the merge rescans all candidate lanes' rows in full
//     precision (usually exactly one lane).
// Rescans use the identical arithmetic, so the keys are exact (distance bits,
// lowest index) before the 128-bit atomic merge across CTAs.
#ifndef TPO_CD_R
#define TPO_CD_R 8
#endif
constexpr int CD_R = TPO_CD_R;   // rows per lane
constexpr int CD_C = 4;          // columns per step (= the row chunk)
constexpr int CD_TILE = 256;
constexpr int CD_W = 4;
constexpr int CD_ROWS_PER_WARP = 32 * CD_R;

__device__ __forceinline__ unsigned hiword(double d) { return (unsigned)__double2hiint(d); }

template <int MODE>
__global__ void __launch_bounds__(CD_W * 32, 2)
    chamfer_keys_f64_kernel(const double* __restrict__ xyz1, const double* __restrict__ xyz2,
                            int64_t N, int64_t M, int64_t row_begin, int64_t row_end,
                            int rb_count, int cs_count, int64_t seg, Key128* __restrict__ keys1,
                            Key128* __restrict__ keys2) {
  using G = GenDist<double, MODE>;
  __shared__ __align__(16) double s_rows[CD_W * CD_ROWS_PER_WARP * 3];
  __shared__ __align__(16) double s_col[CD_TILE][3];
  __shared__ uint2 s_wb[CD_W][CD_TILE];  // {ballot, minimum high word}

  pdl_wait();
  const int W = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int64_t unit = blockIdx.x;
  const int cs = (int)(unit % cs_count);
  unit /= cs_count;
  const int rb = (int)(unit % rb_count);
  const int64_t b = unit / rb_count;
  const int64_t c0 = (int64_t)cs * seg;
  const int64_t c1 = min(M, c0 + seg);
  const int64_t blk_row0 = row_begin + (int64_t)rb * W * CD_ROWS_PER_WARP;
  const int64_t warp_row0 = blk_row0 + (int64_t)warp * CD_ROWS_PER_WARP;
  const int lrow0 = warp * CD_ROWS_PER_WARP + lane * CD_R;  // first row of the lane in s_rows
  const bool warp_active = warp_row0 < row_end;
  const int n_active = (int)min64(W, (row_end - blk_row0 + CD_ROWS_PER_WARP - 1) / CD_ROWS_PER_WARP);
  const double qnan = G::nan_();
  const int64_t nrow = min64((int64_t)W * CD_ROWS_PER_WARP, max64(row_end - blk_row0, 0));
  for (int e = threadIdx.x; e < W * CD_ROWS_PER_WARP * 3; e += blockDim.x)
    s_rows[e] = e < nrow * 3 ? __ldg(xyz1 + (b * N + blk_row0) * 3 + e) : qnan;
  __syncthreads();
  double qx[CD_R], qy[CD_R], qz[CD_R];
#pragma unroll
  for (int r = 0; r < CD_R; ++r) {
    qx[r] = s_rows[(lrow0 + r) * 3];
    qy[r] = s_rows[(lrow0 + r) * 3 + 1];
    qz[r] = s_rows[(lrow0 + r) * 3 + 2];
  }
  unsigned mh[CD_R];
  int bchunk[CD_R];
  unsigned ties = 0;  // bit r: a later chunk reached row r's minimum high word
#pragma unroll
  for (int r = 0; r < CD_R; ++r) {
    mh[r] = 0xffffffffu;
    bchunk[r] = (int)c0;
  }

  for (int64_t tc = c0; tc < c1; tc += CD_TILE) {
    const int ncols = (int)min64(CD_TILE, c1 - tc);
    const int nsteps = (ncols + CD_C - 1) / CD_C;
    __syncthreads();
    for (int e = threadIdx.x; e < nsteps * CD_C * 3; e += blockDim.x)
      (&s_col[0][0])[e] = e < ncols * 3 ? __ldg(xyz2 + (b * M + tc) * 3 + e) : qnan;
    __syncthreads();
    if (warp_active) {
#pragma unroll 2
      for (int s = 0; s < nsteps; ++s) {
        unsigned h[CD_C][CD_R];
#pragma unroll
        for (int c = 0; c < CD_C; ++c) {
          const double cx = s_col[s * CD_C + c][0], cy = s_col[s * CD_C + c][1], cz = s_col[s * CD_C + c][2];
#pragma unroll
          for (int r = 0; r < CD_R; ++r) h[c][r] = hiword(G::d(cx, cy, cz, qx[r], qy[r], qz[r]));
        }
        const int colbase = (int)(tc + s * CD_C);
#pragma unroll
        for (int r = 0; r < CD_R; ++r) {
          const unsigned cm = __vimin3_u32(__vimin3_u32(h[0][r], h[1][r], h[2][r]), h[3][r], 0xffffffffu);
          if (cm < mh[r]) {
            mh[r] = cm;
            bchunk[r] = colbase;
            ties &= ~(1u << r);
          } else if (cm == mh[r]) {
            ties |= 1u << r;
          }
        }
#pragma unroll
        for (int c = 0; c < CD_C; ++c) {
          unsigned m = h[c][0];
#pragma unroll
          for (int r = 1; r + 1 < CD_R; r += 2) m = __vimin3_u32(m, h[c][r], h[c][r + 1]);
          if (CD_R % 2 == 0) m = min(m, h[c][CD_R - 1]);
          const unsigned w = redux_min_u32(m);
          const unsigned bal = __ballot_sync(0xffffffffu, m == w);
          if (lane == 0) s_wb[warp][s * CD_C + c] = make_uint2(bal, w);
        }
      }
    }
    __syncthreads();
    // column merge: exact over every candidate lane (usually one)
    for (int col = threadIdx.x; col < ncols; col += blockDim.x) {
      unsigned bw = s_wb[0][col].y;
      for (int w = 1; w < n_active; ++w) bw = min(bw, s_wb[w][col].y);
      const double cx = s_col[col][0], cy = s_col[col][1], cz = s_col[col][2];
      double bd = qnan;
      int brow = -1;
      for (int w = 0; w < n_active; ++w) {
        if (s_wb[w][col].y != bw) continue;
        unsigned bal = s_wb[w][col].x;
        while (bal) {
          const int ln = __ffs(bal) - 1;
          bal &= bal - 1;
          const int r0 = w * CD_ROWS_PER_WARP + ln * CD_R;
          for (int k = 0; k < CD_R; ++k) {
            const double* q = s_rows + (r0 + k) * 3;
            const double d = G::d(cx, cy, cz, q[0], q[1], q[2]);
            // rows ascend in (warp, lane, k) order: strict '<' keeps the lowest
            if (brow < 0 || d < bd) {
              if (!(d != d)) {
                bd = d;
                brow = r0 + k;
              }
            }
          }
        }
      }
      if (brow >= 0)
        key128_min(keys2 + b * M + tc + col, (u64)__double_as_longlong(bd), (u64)(blk_row0 + brow));
    }
  }
  // rows: exact value and lowest column from the recorded chunk, or from the
  // whole segment when a tie on the high word was seen
  if (warp_active) {
    const double* seg_cols = xyz2 + b * M * 3;
#pragma unroll 1
    for (int r = 0; r < CD_R; ++r) {
      const int64_t row = warp_row0 + (int64_t)lane * CD_R + r;
      if (row >= row_end || mh[r] == 0xffffffffu) continue;
      const bool tie = (ties >> r) & 1u;
      const double* q = s_rows + (lrow0 + r) * 3;
      const int64_t j0 = tie ? c0 : bchunk[r];
      const int64_t j1 = tie ? c1 : min64(c1, (int64_t)bchunk[r] + CD_C);
      double bd = 0.0;
      int64_t bj = -1;
      for (int64_t j = j0; j < j1; ++j) {
        const double* c = seg_cols + j * 3;
        const double d = G::d(__ldg(c), __ldg(c + 1), __ldg(c + 2), q[0], q[1], q[2]);
        if (!(d != d) && (bj < 0 || d < bd)) {
          bd = d;
          bj = j;
        }
      }
      if (bj >= 0) key128_min(keys1 + b * N + row, (u64)__double_as_longlong(bd), (u64)bj);
    }
  }
  pdl_trigger();
}

// ------------------------------- finalize -------------------------------
template <typename T>
struct FinTraits;
template <>
struct FinTraits<float> {
  using K = u64;
  template <int MODE>
  __device__ static bool same(const float* a, const float* c, K key) {
    const float d = dist1f<MODE>(__fsub_rn(c[0], a[0]), __fsub_rn(c[1], a[1]), __fsub_rn(c[2], a[2]));
    return __float_as_uint(d) == (unsigned)(key >> 32);
  }
  __device__ static bool empty(K k) { return k == ~0ull; }
  __device__ static unsigned chunk(K k) { return (unsigned)k; }
  __device__ static float value(K k) { return __uint_as_float((unsigned)(k >> 32)); }
};
template <>
struct FinTraits<__half> {
  using K = u64;
  template <int MODE>
  __device__ static bool same(const __half* a, const __half* c, K key) {
    const float d = __half2float(dist1h(hsub_rn(c[0], a[0]), hsub_rn(c[1], a[1]), hsub_rn(c[2], a[2])));
    return __float_as_uint(d) == (unsigned)(key >> 32);
  }
  __device__ static bool empty(K k) { return k == ~0ull; }
  __device__ static unsigned chunk(K k) { return (unsigned)k; }
  __device__ static __half value(K k) { return __float2half_rn(__uint_as_float((unsigned)(k >> 32))); }
};
template <>
struct FinTraits<double> {
  using K = Key128;
  template <int MODE>
  __device__ static bool same(const double* a, const double* c, K key) {
    const double d = dist1d<MODE>(__dsub_rn(c[0], a[0]), __dsub_rn(c[1], a[1]), __dsub_rn(c[2], a[2]));
    return (u64)__double_as_longlong(d) == key.hi;
  }
  __device__ static bool empty(K k) { return k.hi == ~0ull && k.lo == ~0ull; }
  __device__ static unsigned chunk(K k) { return (unsigned)k.lo; }
  __device__ static double value(K k) { return __longlong_as_double((long long)k.hi); }
};

template <typename T>
struct FinRound {
  __device__ static T from(double v) { return (T)v; }
  __device__ static T add(T a, T b) { return a + b; }
};
template <>
struct FinRound<__half> {
  __device__ static __half from(double v) { return __float2half_rn((float)v); }
  __device__ static __half add(__half a, __half b) { return hadd_rn(a, b); }
};

// Optional fused reduction of the forward (ChamferDistance "mean"/"sum"): each
// block sums its points' distances in a fixed order, writes a partial, and the
// last block to finish adds the partials in block order -- deterministic for a
// given grid.  partials/counter live in the caller's workspace.
template <typename T>
struct FinLoss {
  double* partials;   // 2 per block: sum(dist1), sum(dist2)
  unsigned* counter;  // blocks done, starting from 0xffffffff
  T* loss;            // nullptr: no reduction
  int reduction;      // 0 mean(d1)+mean(d2), 1 sum(d1)+sum(d2)
};

template <typename T>
__device__ __forceinline__ double to_d(T v) { return (double)v; }
template <>
__device__ __forceinline__ double to_d<__half>(__half v) { return (double)__half2float(v); }

// First index in [base, end) whose distance to q has the key's exact bits.  All
// candidate loads are issued before any compare (independent, unrolled), so the
// scan costs one memory round trip instead of one per candidate.
template <typename T, int MODE, int CH, bool Q_IS_ROW>
__device__ __forceinline__ int32_t find_in_chunk(const T* q, const T* cloud, int64_t base,
                                                 int64_t end, typename FinTraits<T>::K key,
                                                 T* xyz = nullptr) {
  T c[CH][3];
  bool loaded = false;
  if constexpr (std::is_same<T, float>::value && CH % 4 == 0) {
    // a whole chunk whose start is 16-byte aligned (chunk starts are multiples
    // of 8 columns, so this holds whenever the cloud itself is aligned): CH*3
    // consecutive floats as float4 loads instead of CH*3 scalar ones
    const float* src = cloud + base * 3;
    if (base + CH <= end && ((uintptr_t)src & 15) == 0) {
      float f[CH * 3];
#pragma unroll
      for (int v = 0; v < CH * 3 / 4; ++v) {
        const float4 w = __ldg(reinterpret_cast<const float4*>(src) + v);
        f[4 * v] = w.x; f[4 * v + 1] = w.y; f[4 * v + 2] = w.z; f[4 * v + 3] = w.w;
      }
#pragma unroll
      for (int k = 0; k < CH; ++k)
#pragma unroll
        for (int d = 0; d < 3; ++d) c[k][d] = f[k * 3 + d];
      loaded = true;
    }
  }
  if (!loaded) {
#pragma unroll
    for (int k = 0; k < CH; ++k) {
      const bool ok = base + k < end;
#pragma unroll
      for (int d = 0; d < 3; ++d) c[k][d] = ok ? cloud[(base + k) * 3 + d] : q[d];
    }
  }
  int found = -1;
#pragma unroll
  for (int k = CH - 1; k >= 0; --k) {
    const bool hit = Q_IS_ROW ? FinTraits<T>::template same<MODE>(q, c[k], key)
                              : FinTraits<T>::template same<MODE>(c[k], q, key);
    if (base + k < end && hit) found = k;
  }
  if (xyz) {  // the found point's coordinates, from the registers already loaded
    found = found < 0 ? 0 : found;
#pragma unroll
    for (int k = 0; k < CH; ++k)
      if (k == found) { xyz[0] = c[k][0]; xyz[1] = c[k][1]; xyz[2] = c[k][2]; }
  }
  return (int32_t)(base + (found < 0 ? 0 : found));
}

// One thread per output point.  Rows: key chunk = first of `row_chunk` columns.
// Columns: key chunk = first of `col_chunk` rows (R of the keys kernel).
// dist1 / dist2 may be null (loss-only use); do_cols selects the column side.
template <typename T, int MODE, int ROWCH, int COLCH>
__global__ void chamfer_finalize_kernel(const T* __restrict__ xyz1, const T* __restrict__ xyz2,
                                        int64_t B, int64_t N, int64_t M, int64_t row_begin,
                                        int64_t row_end,
                                        const typename FinTraits<T>::K* __restrict__ keys1,
                                        const typename FinTraits<T>::K* __restrict__ keys2,
                                        T* __restrict__ dist1, int32_t* __restrict__ idx1,
                                        T* __restrict__ dist2, int32_t* __restrict__ idx2,
                                        bool do_cols, FinLoss<T> fl) {
  using F = FinTraits<T>;
  pdl_wait();
  const int64_t nrows = row_end - row_begin;
  const int64_t n1 = B * nrows;
  const int64_t total = n1 + (do_cols ? B * M : 0);
  double s1 = 0.0, s2 = 0.0;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    if (t < n1) {
      const int64_t b = t / nrows, i = row_begin + t % nrows;
      const int64_t o = b * N + i;
      const typename F::K key = keys1[o];
      T dv = T(0.0f);
      int32_t ix = 0;
      if (M > 0 && !F::empty(key)) {
        const unsigned base = F::chunk(key);
        const T* a = xyz1 + o * 3;
        const T q[3] = {a[0], a[1], a[2]};
        ix = find_in_chunk<T, MODE, ROWCH, true>(q, xyz2 + b * M * 3, base,
                                                 min64(M, (int64_t)base + ROWCH), key);
        dv = F::value(key);
      }
      if (dist1) dist1[o] = dv;
      idx1[o] = ix;
      s1 += to_d(dv);
    } else {
      const int64_t u = t - n1;
      const int64_t b = u / M, j = u % M;
      const int64_t o = b * M + j;
      const typename F::K key = keys2[o];
      T dv = T(0.0f);
      int32_t ix = 0;
      if (N > 0 && !F::empty(key)) {
        const unsigned base = F::chunk(key);
        const T* c = xyz2 + o * 3;
        if constexpr (COLCH == 1) {
          ix = (int32_t)base;  // the keys kernel already stored the exact row
        } else {
          const T q[3] = {c[0], c[1], c[2]};
          ix = find_in_chunk<T, MODE, COLCH, false>(q, xyz1 + b * N * 3, base,
                                                    min64(N, (int64_t)base + COLCH), key);
        }
        dv = F::value(key);
      }
      if (dist2) dist2[o] = dv;
      idx2[o] = ix;
      s2 += to_d(dv);
    }
  }
  if (fl.loss == nullptr) return;
  // block reduction (fixed order), then the last block folds the partials
  __shared__ double r1[32], r2[32];
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    s1 += __shfl_down_sync(0xffffffffu, s1, off);
    s2 += __shfl_down_sync(0xffffffffu, s2, off);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) { r1[warp] = s1; r2[warp] = s2; }
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) {
    double a = 0.0, c = 0.0;
    for (int w = 0; w < nw; ++w) { a += r1[w]; c += r2[w]; }
    fl.partials[2 * blockIdx.x] = a;
    fl.partials[2 * blockIdx.x + 1] = c;
    __threadfence();
    // the counter starts at 0xffffffff (it shares the keys' 0xff fill)
    last = atomicAdd(fl.counter, 1u) == gridDim.x - 2u;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // the last block folds the partials: fixed per-thread strides, then a fixed tree
  double a = 0.0, c = 0.0;
  for (unsigned k = threadIdx.x; k < gridDim.x; k += blockDim.x) {
    a += __ldcg(fl.partials + 2 * k);
    c += __ldcg(fl.partials + 2 * k + 1);
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    a += __shfl_down_sync(0xffffffffu, a, off);
    c += __shfl_down_sync(0xffffffffu, c, off);
  }
  __syncthreads();
  if (lane == 0) { r1[warp] = a; r2[warp] = c; }
  __syncthreads();
  if (threadIdx.x != 0) return;
  a = 0.0;
  c = 0.0;
  for (int w = 0; w < nw; ++w) { a += r1[w]; c += r2[w]; }
  // torch semantics: mean(d1) + mean(d2) (or sums), each term rounded to T, added in T
  T t1, t2;
  if (fl.reduction == 0) {
    t1 = FinRound<T>::from(B * N > 0 ? a / (double)(B * N) : __longlong_as_double(0x7ff8000000000000ll));
    t2 = FinRound<T>::from(B * M > 0 ? c / (double)(B * M) : __longlong_as_double(0x7ff8000000000000ll));
  } else {
    t1 = FinRound<T>::from(a);
    t2 = FinRound<T>::from(c);
  }
  *fl.loss = FinRound<T>::add(t1, t2);
}

// Backward of the fused loss straight from the forward's keys (fp32 / fp16):
// each point takes its neighbour from its key (column keys hold the exact row;
// row keys the first column of an 8-column chunk, rescanned as in finalize),
// then scatters (2g)(p - q) like chamfer_bwd_kernel, with g the loss gradient
// scaled as torch's MeanBackward does (g / count) or unscaled (sum).
template <typename T>
struct FkOps;
template <>
struct FkOps<float> {
  __device__ static float scale(float g, int64_t n, int red) {
    return __fmul_rn(red == 0 ? __fdiv_rn(g, (float)n) : g, 2.0f);
  }
  __device__ static float term(float g, float a, float b) { return __fmul_rn(g, __fsub_rn(a, b)); }
  __device__ static void add(float* p, float v) { atomicAdd(p, v); }
  __device__ static void add3(float* p, const float* v) { red_add3f(p, v[0], v[1], v[2]); }
  __device__ static float neg(float v) { return -v; }
};
template <>
struct FkOps<__half> {
  __device__ static __half scale(__half g, int64_t n, int red) {
    const __half gs = red == 0 ? __float2half_rn(__half2float(g) / (float)n) : g;
    return hmul_rn(gs, __float2half_rn(2.0f));
  }
  __device__ static __half term(__half g, __half a, __half b) { return hmul_rn(g, hsub_rn(a, b)); }
  __device__ static void add(__half* p, __half v) { atomicAdd(p, v); }
  __device__ static void add3(__half* p, const __half* v) { red_add3h(p, v[0], v[1], v[2]); }
  __device__ static __half neg(__half v) { return __hneg(v); }
};

template <typename T, int MODE>
__global__ void chamfer_bwd_from_keys_kernel(const T* __restrict__ xyz1, const T* __restrict__ xyz2,
                                             int64_t B, int64_t N, int64_t M,
                                             const u64* __restrict__ keys1,
                                             const u64* __restrict__ keys2,
                                             const T* __restrict__ grad_loss, int reduction,
                                             T* __restrict__ gx1, T* __restrict__ gx2) {
  using O = FkOps<T>;
  pdl_wait();
  const T g = *grad_loss;
  const T g1 = O::scale(g, B * N, reduction);
  const T g2 = O::scale(g, B * M, reduction);
  const int64_t n1 = B * N;
  const int64_t total = n1 + B * M;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const bool row = t < n1;
    const int64_t u = row ? t : t - n1;
    const int64_t P = row ? N : M, Q = row ? M : N;
    const u64 key = row ? __ldg(keys1 + u) : __ldg(keys2 + u);
    const int64_t b = total <= 0xffffffffll ? (int64_t)((unsigned)u / (unsigned)P) : u / P;
    if (Q == 0 || key == ~0ull) continue;
    const T* own = (row ? xyz1 : xyz2) + u * 3;
    const T* other = (row ? xyz2 : xyz1) + b * Q * 3;
    const T q[3] = {own[0], own[1], own[2]};
    const int64_t base = (unsigned)key;
    constexpr int CH = std::is_same<T, float>::value ? CF_CHUNK : CH_CHUNK;
    T pb[3];  // the neighbour's coordinates (rows: taken from the rescan's loads)
    int32_t j;
    if (row) {
      j = find_in_chunk<T, MODE, CH, true>(q, other, base, min64(Q, base + CH), key, pb);
    } else {
      j = (int32_t)base;
      const T* p = other + (int64_t)j * 3;
      pb[0] = p[0]; pb[1] = p[1]; pb[2] = p[2];
    }
    const T gg = row ? g1 : g2;
    T* ga = (row ? gx1 : gx2) + u * 3;
    T* gb = (row ? gx2 : gx1) + (b * Q + j) * 3;
    T v[3], nv[3];
#pragma unroll
    for (int d = 0; d < 3; ++d) {
      v[d] = O::term(gg, q[d], pb[d]);
      nv[d] = O::neg(v[d]);
    }
    O::add3(ga, v);
    O::add3(gb, nv);
  }
}

// ------------------------------- host side -------------------------------
namespace {

struct Plan {
  int warps, rb_count, cs_count;
  int64_t seg;
  int64_t ctas;
};

// Column-segment count: enough CTAs to fill every SM several times over while
// keeping segments long enough to amortise the per-unit row load / flush.
Plan make_plan(int64_t B, int64_t nrows, int64_t M, int rows_per_warp, int max_warps, int slots) {
  Plan p;
  const int64_t warps_needed = (nrows + rows_per_warp - 1) / rows_per_warp;
  p.warps = (int)std::max<int64_t>(1, std::min<int64_t>(max_warps, warps_needed));
  p.rb_count = (int)((warps_needed + p.warps - 1) / p.warps);
  const int64_t base = B * p.rb_count;
  const int64_t max_cs = std::max<int64_t>(1, (M + 7) / 8);  // segments of >= one 8-column chunk
  // cost model: waves * (columns per unit + fixed overhead in column units)
  double best = 1e300;
  int64_t best_cs = 1;
  const int64_t lim = std::min<int64_t>(max_cs, 4096);
  for (int64_t cs = 1; cs <= lim; ++cs) {
    const int64_t seg = ((M + cs - 1) / cs + 7) / 8 * 8;
    const int64_t real_cs = (M + seg - 1) / seg;
    if (real_cs != cs) continue;
    const int64_t units = base * cs;
    const double waves = (double)((units + slots - 1) / slots);
    const double cost = waves * (double)(seg + 96);
    if (cost < best * 0.999) {
      best = cost;
      best_cs = cs;
    }
  }
  p.seg = std::max<int64_t>(8, ((M + best_cs - 1) / best_cs + 7) / 8 * 8);
  p.cs_count = (int)((M + p.seg - 1) / p.seg);
  p.ctas = base * p.cs_count;
  return p;
}

template <typename KernelT>
int slots_for(KernelT kernel, int threads) {
  int dev = 0;
  cudaGetDevice(&dev);
  int sms = 0, per_sm = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0);
  return std::max(1, sms * std::max(1, per_sm));
}

template <int MODE>
int launch_keys_f32(const float* x1, const float* x2, int64_t B, int64_t N, int64_t M,
                    int64_t rb0, int64_t rb1, void* k1, void* k2, cudaStream_t st) {
  auto kern = chamfer_keys_f32_kernel<MODE>;
  static thread_local int slots_cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int& slots = slots_cache[dev & 63];
  if (!slots) slots = slots_for(kern, CF_MAXW * 32);
  const Plan p = make_plan(B, rb1 - rb0, M, CF_ROWS_PER_WARP, CF_MAXW, slots);
  if (p.ctas <= 0) return TPO_OK;
  return launch_pdl(kern, dim3((unsigned)p.ctas), dim3(p.warps * 32), 0, st, x1, x2, N, M, rb0, rb1,
                    p.rb_count, p.cs_count, p.seg, (u64*)k1, (u64*)k2);
}

int launch_keys_f16(const __half* x1, const __half* x2, int64_t B, int64_t N, int64_t M,
                    int64_t rb0, int64_t rb1, void* k1, void* k2, cudaStream_t st) {
  auto kern = chamfer_keys_f16_kernel;
  static thread_local int slots_cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int& slots = slots_cache[dev & 63];
  if (!slots) slots = slots_for(kern, CF_MAXW * 32);
  const Plan p = make_plan(B, rb1 - rb0, M, CF_ROWS_PER_WARP, CF_MAXW, slots);
  if (p.ctas <= 0) return TPO_OK;
  return launch_pdl(kern, dim3((unsigned)p.ctas), dim3(p.warps * 32), 0, st, x1, x2, N, M, rb0, rb1,
                    p.rb_count, p.cs_count, p.seg, (u64*)k1, (u64*)k2);
}

template <int MODE>
int launch_keys_f64(const double* x1, const double* x2, int64_t B, int64_t N, int64_t M, int64_t rb0,
                    int64_t rb1, void* k1, void* k2, cudaStream_t st) {
  auto kern = chamfer_keys_f64_kernel<MODE>;
  static thread_local int slots_cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int& slots = slots_cache[dev & 63];
  if (!slots) slots = slots_for(kern, CD_W * 32);
  const Plan p = make_plan(B, rb1 - rb0, M, CD_ROWS_PER_WARP, CD_W, slots);
  if (p.ctas <= 0) return TPO_OK;
  return launch_pdl(kern, dim3((unsigned)p.ctas), dim3(p.warps * 32), 0, st, x1, x2, N, M, rb0, rb1,
                    p.rb_count, p.cs_count, p.seg, (Key128*)k1, (Key128*)k2);
}

template <typename T, int MODE, int ROWCH, int COLCH>
int launch_finalize(const T* x1, const T* x2, int64_t B, int64_t N, int64_t M, int64_t rb0,
                    int64_t rb1, const void* k1, const void* k2,
                    T* d1, int32_t* i1, T* d2, int32_t* i2, bool do_cols, T* loss,
                    int reduction, void* loss_ws, cudaStream_t st) {
  const int64_t total = B * (rb1 - rb0) + (do_cols ? B * M : 0);
  if (total <= 0 && loss == nullptr) return TPO_OK;
  const int threads = 256;
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((total + threads - 1) / threads,
                                                                 kFinMaxBlocks));
  FinLoss<T> fl;
  fl.loss = loss;
  fl.reduction = reduction;
  fl.partials = (double*)loss_ws;
  fl.counter = loss_ws ? (unsigned*)((char*)loss_ws + kFinPartialBytes) : nullptr;
  return launch_pdl(chamfer_finalize_kernel<T, MODE, ROWCH, COLCH>, dim3((unsigned)blocks), dim3(threads), 0,
                    st, x1, x2, B, N, M, rb0, rb1, (const typename FinTraits<T>::K*)k1,
                    (const typename FinTraits<T>::K*)k2, d1, i1, d2, i2, do_cols, fl);
}

}  // namespace

int chamfer_fwd_keys(int dtype, int flags, const void* x1, const void* x2, int64_t B, int64_t N,
                     int64_t M, int64_t rb0, int64_t rb1, void* k1, void* k2, cudaStream_t st) {
  const bool exact = (flags & TPO_ROUND_EXACT) != 0;
  if (B == 0 || rb1 <= rb0 || M == 0) return TPO_OK;
  switch (dtype) {
    case TPO_F32:
      return exact ? launch_keys_f32<TPO_ROUND_EXACT>((const float*)x1, (const float*)x2, B, N, M, rb0, rb1, k1, k2, st)
                   : launch_keys_f32<TPO_ROUND_FMA>((const float*)x1, (const float*)x2, B, N, M, rb0, rb1, k1, k2, st);
    case TPO_F16:
      return launch_keys_f16((const __half*)x1, (const __half*)x2, B, N, M, rb0, rb1, k1, k2, st);
    case TPO_F64:
      return exact ? launch_keys_f64<TPO_ROUND_EXACT>((const double*)x1, (const double*)x2, B, N, M, rb0, rb1, k1, k2, st)
                   : launch_keys_f64<TPO_ROUND_FMA>((const double*)x1, (const double*)x2, B, N, M, rb0, rb1, k1, k2, st);
  }
  return TPO_ERR_INVALID_ARGUMENT;
}

int chamfer_finalize(int dtype, int flags, const void* x1, const void* x2, int64_t B, int64_t N,
                     int64_t M, int64_t rb0, int64_t rb1, const void* k1, const void* k2, void* d1,
                     int32_t* i1, void* d2, int32_t* i2, bool do_cols, void* loss, int reduction,
                     void* loss_ws, cudaStream_t st) {
  const bool exact = (flags & TPO_ROUND_EXACT) != 0;
#define TPO_FIN(T, MODE, CH, CC)                                                                 \
  launch_finalize<T, MODE, CH, CC>((const T*)x1, (const T*)x2, B, N, M, rb0, rb1, k1, k2, (T*)d1, \
                           i1, (T*)d2, i2, do_cols, (T*)loss, reduction, loss_ws, st)
  switch (dtype) {
    case TPO_F32:
      return exact ? TPO_FIN(float, TPO_ROUND_EXACT, CF_CHUNK, 1) : TPO_FIN(float, TPO_ROUND_FMA, CF_CHUNK, 1);
    case TPO_F16:
      return TPO_FIN(__half, TPO_ROUND_EXACT, CH_CHUNK, 1);
    case TPO_F64:
      return exact ? TPO_FIN(double, TPO_ROUND_EXACT, CG_C, CG_R) : TPO_FIN(double, TPO_ROUND_FMA, CG_C, CG_R);
  }
#undef TPO_FIN
  return TPO_ERR_INVALID_ARGUMENT;
}

// Loss from the final keys in a separate small kernel: grid-stride sums of the
// row and column distances (fixed per-thread order), block partials, and the
// last block folds them in block order -- deterministic for a given grid.
// Cheaper than the keys kernel's per-batch last-CTA epilogue, whose serial
// chain of counter atomics and loads sat at the end of the critical path.
__global__ void keys_loss_reduce_kernel(const u64* __restrict__ k1, int64_t n1,
                                        const u64* __restrict__ k2, int64_t n2,
                                        double* __restrict__ part, unsigned* ctr, void* loss,
                                        int half_out, int reduction) {
  __shared__ double sa[32], sc[32];
  pdl_wait();
  double a = 0.0, c = 0.0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n1;
       i += (int64_t)gridDim.x * blockDim.x)
    a += (double)__uint_as_float((unsigned)(__ldg(k1 + i) >> 32));
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n2;
       i += (int64_t)gridDim.x * blockDim.x)
    c += (double)__uint_as_float((unsigned)(__ldg(k2 + i) >> 32));
  block_sum2(a, c, sa, sc);
  __shared__ bool s_last;
  if (threadIdx.x == 0) {
    __stcg(part + 2 * blockIdx.x, a);
    __stcg(part + 2 * blockIdx.x + 1, c);
    s_last = atom_add_acq_rel(ctr, 1u) == gridDim.x - 2u;  // counter starts at 0xffffffff
  }
  __syncthreads();
  if (!s_last) return;
  a = 0.0;
  c = 0.0;
  for (unsigned k = threadIdx.x; k < gridDim.x; k += blockDim.x) {
    a += __ldcg(part + 2 * k);
    c += __ldcg(part + 2 * k + 1);
  }
  block_sum2(a, c, sa, sc);
  if (threadIdx.x != 0) return;
  const double v1 = reduction == 0 ? a / (double)n1 : a;
  const double v2 = reduction == 0 ? c / (double)n2 : c;
  if (half_out)
    *(__half*)loss = hadd_rn(__float2half_rn((float)v1), __float2half_rn((float)v2));
  else
    *(float*)loss = __fadd_rn((float)v1, (float)v2);
}

int chamfer_loss_keys(int dtype, int flags, const void* x1, const void* x2, int64_t B, int64_t N,
                      int64_t M, int reduction, void* k1, void* k2, void* lossws, void* loss,
                      void* partials, cudaStream_t st) {
  int s;
  if (dtype == TPO_F16)
    s = launch_keys_f16((const __half*)x1, (const __half*)x2, B, N, M, 0, N, k1, k2, st);
  else if (flags & TPO_ROUND_EXACT)
    s = launch_keys_f32<TPO_ROUND_EXACT>((const float*)x1, (const float*)x2, B, N, M, 0, N, k1, k2, st);
  else
    s = launch_keys_f32<TPO_ROUND_FMA>((const float*)x1, (const float*)x2, B, N, M, 0, N, k1, k2, st);
  if (s) return s;
  const int threads = 256;
  const int64_t want = (B * (N + M) + threads * 8 - 1) / (threads * 8);
  const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>(want, 296));
  unsigned* ctr = (unsigned*)lossws + B;  // the 0xff-filled counter word after the batch counters
  return launch_pdl(keys_loss_reduce_kernel, dim3(blocks), dim3(threads), 0, st, (const u64*)k1, B * N,
                    (const u64*)k2, B * M, (double*)partials, ctr, loss, (int)(dtype == TPO_F16),
                    reduction);
}

int chamfer_bwd_from_keys(int dtype, int flags, const void* x1, const void* x2, int64_t B,
                          int64_t N, int64_t M, const void* k1, const void* k2,
                          const void* grad_loss, int reduction, void* gx1, void* gx2,
                          cudaStream_t st) {
  const int64_t total = B * (N + M);
  if (total <= 0) return TPO_OK;
  const int threads = 256;
  const unsigned blocks = (unsigned)std::min<int64_t>((total + threads - 1) / threads, 148 * 16);
  const bool exact = (flags & TPO_ROUND_EXACT) != 0;
  const u64* K1 = (const u64*)k1;
  const u64* K2 = (const u64*)k2;
  if (dtype == TPO_F16)
    return launch_pdl(chamfer_bwd_from_keys_kernel<__half, TPO_ROUND_EXACT>, dim3(blocks), dim3(threads), 0, st,
                      (const __half*)x1, (const __half*)x2, B, N, M, K1, K2, (const __half*)grad_loss,
                      reduction, (__half*)gx1, (__half*)gx2);
  if (exact)
    return launch_pdl(chamfer_bwd_from_keys_kernel<float, TPO_ROUND_EXACT>, dim3(blocks), dim3(threads), 0, st,
                      (const float*)x1, (const float*)x2, B, N, M, K1, K2, (const float*)grad_loss,
                      reduction, (float*)gx1, (float*)gx2);
  return launch_pdl(chamfer_bwd_from_keys_kernel<float, TPO_ROUND_FMA>, dim3(blocks), dim3(threads), 0, st,
                    (const float*)x1, (const float*)x2, B, N, M, K1, K2, (const float*)grad_loss,
                    reduction, (float*)gx1, (float*)gx2);
}

int device_error_flags(unsigned* out, bool clear) {
  int s = cuda_status(cudaMemcpyFromSymbol(out, g_fwd_device_error, sizeof(unsigned)));
  if (s || !clear) return s;
  const unsigned zero = 0;
  return cuda_status(cudaMemcpyToSymbol(g_fwd_device_error, &zero, sizeof(unsigned)));
}

}  // namespace tpo
