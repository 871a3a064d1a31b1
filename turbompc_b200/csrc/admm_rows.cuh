// Fused ADMM solve with register-resident operators: stage blocks of width 16
// (n <= 16), fp32, horizons up to T = 64 (the quadrotor configuration has
// n = 16, T = 51; the Clohessy-Wiltshire one n = 9, T = 61).
//
// Same algorithm and iteration order as admm_fused_kernel (admm_kernel.cuh);
// only the linear-system layer differs.  Eight threads own one stage block t,
// thread q owning rows q and q + 8, and keep in registers
//   Theta_t^-1 rows        (16 + 16 values)
//   S(t, t-1) = Phi_{t-1}  rows
//   S(t, t+1) = Phi_t^T    rows (= columns of Phi_t)
// so every product is a row-times-vector with the vector broadcast from
// shared memory and every output row is produced by the thread that owns it:
// no partial-sum buffers and no cross-thread reductions inside a matvec.
// Only the diagonal blocks Theta_t of S stay in shared memory.
//
// The block-tridiagonal preconditioner of the reference (admm.py:123-153)
//   Phiinv = blocktridiag(Theta_t^-1 Phi_{t-1} Theta_{t-1}^-1, -Theta_t^-1,
//                         Theta_t^-1 Phi_t^T Theta_{t+1}^-1)
// equals Dth (Phi_off - Theta) Dth with Dth = blockdiag(Theta_t^-1) and
// Phi_off the off-diagonal part of S, so it is applied in factored form:
//   w = Dth r ;  u = Phi_off w ;  z = Dth u - w
// which needs no storage beyond S's blocks and Theta^-1 (the same operator up
// to rounding; parity is checked at the fp32 tolerance).
#pragma once

#include "admm_kernel.cuh"

namespace tmpc {

// Optional phase timers (build with -DTMPC_ROWS_PROFILE): thread 0 of every
// CTA adds the clock64 cycles of each phase to g_rows_prof, read back with
// tmpc_debug_rows_profile.  Compiled out of the regular library.
#ifdef TMPC_ROWS_PROFILE
__device__ unsigned long long g_rows_prof[16];
#define TMPC_PROF_INIT long long prof_t0_ = clock64();
#define TMPC_PROF(k)                                                   \
  do {                                                                 \
    if (threadIdx.x == 0) {                                            \
      const long long now_ = clock64();                                \
      atomicAdd(&g_rows_prof[k], (unsigned long long)(now_ - prof_t0_)); \
      prof_t0_ = now_;                                                 \
    }                                                                  \
  } while (0)
#else
#define TMPC_PROF_INIT
#define TMPC_PROF(k) \
  do {               \
  } while (0)
#endif

struct RowsGeo {
  static constexpr int NB = 16;
  static constexpr int TPB = 8;           // threads per stage block
  static constexpr int VSTR = 20;         // block-vector row stride (80 B: odd multiple of 16 B)
  static constexpr int BSTR = 24;         // broadcast-buffer row stride: 8-word windows of 4 consecutive
                                          // stages land on disjoint banks (24 t mod 32 = 0, 24, 16, 8)
  static constexpr int TSTR = 20;         // row stride of a Theta block in shared memory
  static constexpr int TBLK = 16 * TSTR;  // Theta block stride
  static constexpr int SQ = 256;          // dense 16 x 16 scratch block
  static constexpr int TMAX = 64;  // largest horizon + 1 (two instances: 52 and 64 stages)
};
// Stage capacity of the kernel instance that runs T stages: 52 (the quadrotor
// size, 416 threads) or 64 (512 threads; 128 registers per thread either way).
// The broadcast buffers are sized by the capacity, and the 64-stage instance's
// larger buffers would push the 52-stage problems past the shared-memory limit.
__host__ __device__ constexpr int rows_cap(int T) { return T <= 52 ? 52 : 64; }
// One broadcast buffer (zero rows around the stages) for capacity TM.
__host__ __device__ constexpr int rows_buf(int TM) { return (TM + 3) * RowsGeo::BSTR; }
static_assert(Geo<16, float>::VSTR == RowsGeo::VSTR, "block-vector stride shared with the ADMM helpers");

__host__ __device__ constexpr int rows_threads(int T) { return (T * RowsGeo::TPB + 31) / 32 * 32; }
__host__ __device__ constexpr int rows_tpad(int T) { return rows_threads(T) / RowsGeo::TPB; }

// Element offsets inside the dynamic shared-memory arena.  The four broadcast
// buffers (p, w, r, u) have a zero row before stage 0 and zero rows after
// stage T-1, so row index t + 1 holds stage t and neighbours need no bounds
// tests.
struct RowsSmem {
  // stage: a copy of the QP data the assembly and the ADMM-level steps read
  // (q, A0, Am, Ap, G, c0, c, l, u); tslot: one 16 x 16 block per warp for
  // handing -Theta_t^-1 from the Gauss-Jordan warp to the block's owners.
  size_t th, stage, sq, sa0, sam, sap, sg, sc0, sc, sl, su, tslot, bb, x, gam, xold, yf0, yfd, zg, yg, xig, red,
      nelem;
  RowsSmem() = default;
  __host__ __device__ RowsSmem(int T, int n, int nx, int n0, int m, int buf) {
    using G = RowsGeo;
    const int N = T - 1, TP = rows_tpad(T);
    auto a4 = [](size_t v) { return (v + 3) & ~size_t(3); };
    size_t o = 0;
    th = o; o += (size_t)TP * G::TBLK;
    stage = o;
    sq = o; o = a4(o + (size_t)T * n);
    sa0 = o; o = a4(o + (size_t)n0 * n);
    sam = o; o = a4(o + (size_t)N * nx * n);
    sap = o; o = a4(o + (size_t)N * nx * n);
    sg = o; o = a4(o + (size_t)T * m * n);
    sc0 = o; o = a4(o + n0);
    sc = o; o = a4(o + (size_t)N * nx);
    sl = o; o = a4(o + (size_t)T * m);
    su = o; o = a4(o + (size_t)T * m);
    tslot = o; o += (size_t)(rows_threads(T) / 32) * G::SQ;
    bb = o; o += 4 * (size_t)buf;  // p, w, r, u broadcast buffers at constant offsets
    x = o; o += (size_t)T * G::VSTR;
    gam = o; o += (size_t)T * G::VSTR;
    xold = o; o += (size_t)T * G::VSTR;
    yf0 = a4(o); o = yf0 + n0;
    yfd = a4(o); o = yfd + (size_t)N * nx;
    zg = a4(o); o = zg + (size_t)T * m;
    yg = a4(o); o = yg + (size_t)T * m;
    xig = a4(o); o = xig + (size_t)T * m;
    red = a4(o); o = red + kRedSize;  // residual table and scalars, 2 x 16 dot slots
    nelem = a4(o);
  }
};

// Copies the per-iteration QP data of one problem into the stage area (D and
// E stay in global memory: only the residual checks read them).
__device__ __forceinline__ void rows_stage_qp(float* sm, const RowsSmem& L, const QPView<float>& g, int T,
                                                       int n, int nx, int n0, int m) {
  const int N = T - 1;
  auto copy = [](float* dst, const float* src, int cnt) {
    if (src == nullptr) return;
    if ((cnt & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
#pragma unroll 4
      for (int e = threadIdx.x; e < cnt / 4; e += blockDim.x)
        reinterpret_cast<float4*>(dst)[e] = __ldg(reinterpret_cast<const float4*>(src) + e);
    } else {
      for (int e = threadIdx.x; e < cnt; e += blockDim.x) dst[e] = __ldg(src + e);
    }
  };
  copy(sm + L.sq, g.q, T * n);
  copy(sm + L.sa0, g.A0, n0 * n);
  copy(sm + L.sam, g.Am, N * nx * n);
  copy(sm + L.sap, g.Ap, N * nx * n);
  copy(sm + L.sg, g.G, T * m * n);
  copy(sm + L.sc0, g.c0, n0);
  copy(sm + L.sc, g.c, N * nx);
  copy(sm + L.sl, g.l, T * m);
  copy(sm + L.su, g.u, T * m);
}

// Gauss-Jordan source / destination: Theta from its shared-memory blocks,
// -Theta_t^-1 into the slot of the warp that inverts it (t - base).
struct RowsInvAcc {
  const float* th;
  float* tslot;
  int base;
  __device__ float get_theta(int t, int i, int j) const { return th[t * RowsGeo::TBLK + i * RowsGeo::TSTR + j]; }
  __device__ void set_ntinv(int t, int i, int j, float v) const {
    float* b = tslot + (t - base) * RowsGeo::SQ;
    b[i * 16 + j] = v;
    b[j * 16 + i] = v;
  }
};

struct RowOps {
  float2 ti[2][8];  // Theta_t^-1 rows q, q + 8, as column pairs (2c, 2c + 1)
  float2 lr[2][8];  // S(t, t-1) rows
  float2 lc[2][8];  // S(t, t+1) rows
};

// The block-row products use the paired FP32 FMA of sm_100 (FFMA2 through
// __ffma2_rn): each row keeps two partial sums, one over the even and one
// over the odd columns, so a 16-entry row costs eight paired FMAs and one add
// instead of sixteen FMAs, and the dependent chain is eight long.  A float4 of
// the broadcast vector supplies the column pairs (2c, 2c + 1) directly.
__device__ __forceinline__ float2 f2lo(const float4 w) { return make_float2(w.x, w.y); }
__device__ __forceinline__ float2 f2hi(const float4 w) { return make_float2(w.z, w.w); }

// a_i = m_i . v for the two owned rows; v is a broadcast 16-vector in shared memory.
__device__ __forceinline__ void rows_bdot(float& a0, float& a1, const float2 (&m0)[8], const float2 (&m1)[8],
                                          const float* v) {
  float2 e0 = make_float2(0.f, 0.f), e1 = make_float2(0.f, 0.f);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float4 w = *reinterpret_cast<const float4*>(v + 4 * c);
    e0 = __ffma2_rn(m0[2 * c], f2lo(w), e0);
    e1 = __ffma2_rn(m1[2 * c], f2lo(w), e1);
    e0 = __ffma2_rn(m0[2 * c + 1], f2hi(w), e0);
    e1 = __ffma2_rn(m1[2 * c + 1], f2hi(w), e1);
  }
  a0 = e0.x + e0.y;
  a1 = e1.x + e1.y;
}

// Same as rows_bdot with four partial sums per row (column pairs 0-3 and
// 4-7 kept apart) for the latency-critical preconditioner steps.
__device__ __forceinline__ void rows_bdot_split(float& a0, float& a1, const float2 (&m0)[8], const float2 (&m1)[8],
                                                const float* v) {
  float2 e0 = make_float2(0.f, 0.f), e1 = make_float2(0.f, 0.f);
  float2 o0 = make_float2(0.f, 0.f), o1 = make_float2(0.f, 0.f);
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const float4 w = *reinterpret_cast<const float4*>(v + 4 * c);
    const float4 u = *reinterpret_cast<const float4*>(v + 8 + 4 * c);
    e0 = __ffma2_rn(m0[2 * c], f2lo(w), e0);
    e1 = __ffma2_rn(m1[2 * c], f2lo(w), e1);
    o0 = __ffma2_rn(m0[4 + 2 * c], f2lo(u), o0);
    o1 = __ffma2_rn(m1[4 + 2 * c], f2lo(u), o1);
    e0 = __ffma2_rn(m0[2 * c + 1], f2hi(w), e0);
    e1 = __ffma2_rn(m1[2 * c + 1], f2hi(w), e1);
    o0 = __ffma2_rn(m0[5 + 2 * c], f2hi(u), o0);
    o1 = __ffma2_rn(m1[5 + 2 * c], f2hi(u), o1);
  }
  a0 = (e0.x + e0.y) + (o0.x + o0.y);
  a1 = (e1.x + e1.y) + (o1.x + o1.y);
}

// Same as rows_bdot with the two matrix rows read from shared memory (Theta rows).
__device__ __forceinline__ void rows_sdot(float& a0, float& a1, const float* r0, const float* r1, const float* v) {
  float2 e0 = make_float2(0.f, 0.f), e1 = make_float2(0.f, 0.f);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float4 w = *reinterpret_cast<const float4*>(v + 4 * c);
    const float4 m0 = *reinterpret_cast<const float4*>(r0 + 4 * c);
    const float4 m1 = *reinterpret_cast<const float4*>(r1 + 4 * c);
    e0 = __ffma2_rn(f2lo(m0), f2lo(w), e0);
    e1 = __ffma2_rn(f2lo(m1), f2lo(w), e1);
    e0 = __ffma2_rn(f2hi(m0), f2hi(w), e0);
    e1 = __ffma2_rn(f2hi(m1), f2hi(w), e1);
  }
  a0 = e0.x + e0.y;
  a1 = e1.x + e1.y;
}

// y = (S v) at the owned rows; vt points at row t of the buffer holding v
// (row t + 1 is stage t).
__device__ __forceinline__ void rows_smv(float (&y)[2], const RowOps& o, const float* th_row, const float* vt) {
  float l0, l1, d0, d1, u0, u1;
  rows_bdot(l0, l1, o.lr[0], o.lr[1], vt);
  rows_sdot(d0, d1, th_row, th_row + 8 * RowsGeo::TSTR, vt + RowsGeo::BSTR);
  rows_bdot(u0, u1, o.lc[0], o.lc[1], vt + 2 * RowsGeo::BSTR);
  y[0] = (l0 + d0) + u0;
  y[1] = (l1 + d1) + u1;
}

// y = (S z) at the owned rows for z = Phiinv r, without Theta: with
// w = Theta^-1 r and f = F w (F: the off-diagonal blocks of S), z = Theta^-1 f - w,
// so Theta z = f - r and S z = (f - r) + F z.  f comes from rows_prec; only
// the two off-diagonal block products of z remain (Theta's rows are not
// read).  The identity holds up to the rounding of Theta^-1 (Theta Theta^-1 =
// I): with the quadrotor QPs (cond(Theta) ~ 1e3) the fp32 PCG iterate after
// 30 iterations differs from the fp64 one by 2e-5 relative with it and by
// 7e-6 with the explicit Theta product.
__device__ __forceinline__ void rows_smv_prec(float (&y)[2], const RowOps& o, const float* vt, const float (&fw)[2],
                                              const float (&r)[2]) {
  float l0, l1, u0, u1;
  rows_bdot(l0, l1, o.lr[0], o.lr[1], vt);
  rows_bdot(u0, u1, o.lc[0], o.lc[1], vt + 2 * RowsGeo::BSTR);
  y[0] = (l0 + (fw[0] - r[0])) + u0;
  y[1] = (l1 + (fw[1] - r[1])) + u1;
}

// z = Phiinv r in factored form.  bt points at row t (stage t - 1) of the p
// buffer; the r, w, u buffers follow at constant offsets.  Contains one
// __syncthreads (all threads call it).
template <int BUF>
__device__ __forceinline__ void rows_prec(float (&z)[2], float (&fw)[2], const float (&r)[2], const RowOps& o, float* bt,
                                          int q) {
  constexpr int VS = RowsGeo::BSTR;
  float* wb = bt + BUF;      // row t of the w buffer
  float* rrow = bt + 2 * BUF + VS;
  float* urow = bt + 3 * BUF + VS;
  rrow[q] = r[0];
  rrow[q + 8] = r[1];
  __syncwarp();  // the eight threads of a stage block share a warp
  float w0, w1;
  rows_bdot_split(w0, w1, o.ti[0], o.ti[1], rrow);
  float* wrow = wb + VS;
  wrow[q] = w0;
  wrow[q + 8] = w1;
  __syncthreads();
  float a0, a1, b0, b1;
  rows_bdot(a0, a1, o.lr[0], o.lr[1], wb);
  rows_bdot(b0, b1, o.lc[0], o.lc[1], wb + 2 * VS);
  fw[0] = a0 + b0;
  fw[1] = a1 + b1;
  urow[q] = fw[0];
  urow[q + 8] = fw[1];
  __syncwarp();
  float v0, v1;
  rows_bdot_split(v0, v1, o.ti[0], o.ti[1], urow);
  z[0] = v0 - w0;
  z[1] = v1 - w1;
}

// The operator rows of a thread are written by rows_build (a call that
// receives the area's address, so the area lives in per-thread local memory,
// L1/L2 backed) and loaded at the start of every PCG solve with 128-bit
// loads, so they occupy registers only inside the PCG loop and the
// ADMM-level steps around it get the register file.
struct __align__(16) RowOpsSave {
  float v[96];  // ti rows (0..31), lr rows (32..63), lc rows (64..95)
  __device__ __forceinline__ void load(RowOps& o) const {
    const float4* p = reinterpret_cast<const float4*>(v);
#pragma unroll
    for (int c = 0; c < 24; ++c) {
      const float4 w = p[c];
      float2* dst = c < 8 ? &o.ti[c >> 2][(c & 3) * 2] : (c < 16 ? &o.lr[(c - 8) >> 2][(c & 3) * 2]
                                                                : &o.lc[(c - 16) >> 2][(c & 3) * 2]);
      dst[0] = f2lo(w);
      dst[1] = f2hi(w);
    }
  }
};

// Two deterministic block sums with one barrier: each warp's sums go to 16
// slots per sum (unused slots stay zero); slots holds 2 x 16 entries.
__device__ __forceinline__ void rows_block_sum2(float& a, float& b, float* slots) {
  a = warp_sum(a);
  b = warp_sum(b);
  if ((threadIdx.x & 31) == 0) {
    slots[threadIdx.x >> 5] = a;
    slots[16 + (threadIdx.x >> 5)] = b;
  }
  __syncthreads();
  // Every thread reads all 16 slots of each sum (broadcast 128-bit loads) and
  // adds them in the same fixed tree order: deterministic and identical in
  // all threads, without the shuffle round trips on the iteration's chain.
  const float4* sl = reinterpret_cast<const float4*>(slots);
  float4 v[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) v[c] = sl[c];
  auto tree16 = [](const float4* w) {
    const float q0 = (w[0].x + w[0].y) + (w[0].z + w[0].w);
    const float q1 = (w[1].x + w[1].y) + (w[1].z + w[1].w);
    const float q2 = (w[2].x + w[2].y) + (w[2].z + w[2].w);
    const float q3 = (w[3].x + w[3].y) + (w[3].z + w[3].w);
    return (q0 + q1) + (q2 + q3);
  };
  a = tree16(v);
  b = tree16(v + 4);
}

// PCG in the single-reduction (Chronopoulos-Gear) arrangement: the same
// iterates as admm_fused.cu:54-161 in exact arithmetic, with both inner
// products of an iteration in one reduction.  With u = M r and w = S u,
//   gamma = r.u, delta = w.u, beta = gamma_new / gamma,
//   p.Sp = delta - beta gamma_new / alpha  (denominator, clamped at 1e-30 as
//   the reference's p.Sp), alpha = gamma_new / (p.Sp),
//   p = u + beta p, s (= S p) = w + beta s, x += alpha p, r -= alpha s.
// The stopping test |gamma| < 1e-12 + eps |gamma_0| runs before each update,
// as the reference's |eta| test, so the iteration counts agree.  Three CTA
// barriers and one reduction per iteration instead of four and two.  w = S u
// is formed without Theta (rows_smv_prec); the initial residual uses the
// explicit S x.  xs /
// gam are [T][VSTR] block vectors in shared memory; x is read from and
// written back to xs.  Returns the iteration count.
template <int BUF>
__device__ __forceinline__ int rows_pcg_cg(const RowOpsSave& saved, const float* th, float* bb, float* xs,
                                           const float* gam, int T, int max_iter, float eps, float* slots) {
  constexpr int VS = RowsGeo::VSTR;
  RowOps o;
  saved.load(o);
  const int t = threadIdx.x >> 3, q = threadIdx.x & 7;
  const bool act = t < T;
  const float* th_row = th + t * RowsGeo::TBLK + q * RowsGeo::TSTR;
  float* bt = bb + t * RowsGeo::BSTR;
  float* prow = bt + RowsGeo::BSTR;
  float x[2], r[2], p[2], sv[2], u[2], w[2];
  x[0] = act ? xs[t * VS + q] : 0.f;
  x[1] = act ? xs[t * VS + q + 8] : 0.f;
  prow[q] = x[0];
  prow[q + 8] = x[1];
  __syncthreads();
  rows_smv(w, o, th_row, bt);
  r[0] = (act ? gam[t * VS + q] : 0.f) - w[0];
  r[1] = (act ? gam[t * VS + q + 8] : 0.f) - w[1];
  float fw[2];
  rows_prec<BUF>(u, fw, r, o, bt, q);  // its barrier ends every read of x in the buffer
  prow[q] = u[0];
  prow[q + 8] = u[1];
  __syncthreads();
  rows_smv_prec(w, o, bt, fw, r);
  float gamma = fmaf(r[1], u[1], r[0] * u[0]);
  float delta = fmaf(w[1], u[1], w[0] * u[0]);
  rows_block_sum2(gamma, delta, slots);
  const float eta0 = fabsf(gamma);
  float den = fabsf(delta) < 1e-30f ? 1e-30f : delta;
  float alpha = gamma / den;
  // Reciprocals 1 / gamma and 1 / alpha for the next iteration's beta and
  // p.Sp, computed here so that alpha = gamma_new / (p.Sp) is the only
  // division on the iteration's dependent chain.
  float rgam = 1.f / gamma;
  float ralpha = den * rgam;
  p[0] = u[0];
  p[1] = u[1];
  sv[0] = w[0];
  sv[1] = w[1];
  int it = 0;
  for (; it < max_iter; ++it) {
    if (fabsf(gamma) < 1e-12f + eps * eta0) break;
    x[0] = fmaf(alpha, p[0], x[0]);
    x[1] = fmaf(alpha, p[1], x[1]);
    r[0] = fmaf(-alpha, sv[0], r[0]);
    r[1] = fmaf(-alpha, sv[1], r[1]);
    rows_prec<BUF>(u, fw, r, o, bt, q);  // its barrier ends every read of the previous u
    prow[q] = u[0];
    prow[q + 8] = u[1];
    __syncthreads();
    rows_smv_prec(w, o, bt, fw, r);
    float gnew = fmaf(r[1], u[1], r[0] * u[0]);
    float dl = fmaf(w[1], u[1], w[0] * u[0]);
    rows_block_sum2(gnew, dl, slots);
    const float beta = gnew * rgam;
    float pap = dl - beta * gnew * ralpha;
    if (fabsf(pap) < 1e-30f) pap = 1e-30f;
    alpha = gnew / pap;
    gamma = gnew;
    rgam = 1.f / gnew;  // off the chain: used from the next iteration on
    ralpha = pap * rgam;
    p[0] = fmaf(beta, p[0], u[0]);
    p[1] = fmaf(beta, p[1], u[1]);
    sv[0] = fmaf(beta, sv[0], w[0]);
    sv[1] = fmaf(beta, sv[1], w[1]);
  }
  if (act) {
    xs[t * VS + q] = x[0];
    xs[t * VS + q + 8] = x[1];
  }
  __syncthreads();
  return it;
}


// Operator build for one rho (the math of admm.py:71-154, restated per owner
// thread).  Thread (t, q) computes rows q and q + 8 of every block it owns:
//   Theta_t rows      D + sigma I + rho G^T G + rho_f (A^T A terms), from the
//                     staged QP (rows of the A / G blocks broadcast from shared
//                     memory), stored to shared memory for the S-matvec;
//   Theta_t^-1 rows   Gauss-Jordan on [Theta_t | I] by the stage's eight
//                     threads (one warp), pivot rows exchanged through shared
//                     memory; Theta_t is symmetric positive definite, so the
//                     elimination runs without row exchanges (the reference
//                     inverts with pivoting, admm_math.cuh:248-310; the results
//                     agree to rounding);
//   Phi_{t-1} rows / Phi_t columns   E + rho_f Ap^T Am, in the reference's
//                     summation order over the constraint rows.
// Every thread's rows go to its save area.  Not inlined (its own register
// allocation).  Ends with a barrier.
__device__ __noinline__ void rows_build(float* sm, const RowsSmem* Lp, const QPView<float> qg,
                                        const QPView<float> qs, float rho_f, float rho, float sigma, int T, int n,
                                        int nx, int n0, int m, int* flag, RowOpsSave* save) {
  const RowsSmem& L = *Lp;
  float* th = sm + L.th;
  const int N = T - 1;
  const int t = threadIdx.x >> 3, q = threadIdx.x & 7;
  const bool act = t < T;
  const int tt = act ? t : 0;
  TMPC_PROF_INIT
  // Row k (n entries, zero padded to 16) of a staged block, broadcast to the stage's threads.
  auto row16 = [&](float (&r)[16], const float* p) {
#pragma unroll
    for (int j = 0; j < 16; ++j) r[j] = j < n ? p[j] : 0.f;
  };
  // ---- Theta rows i = q + 8a
  float a0[16], a1[16];  // [Theta | .] rows, later the Gauss-Jordan rows
  {
    float acc0[16], acc1[16], r[16];
    const int i0 = q, i1 = q + 8;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      a0[j] = (act && i0 < n && j < n) ? qg.D[((size_t)tt * n + i0) * n + j] : 0.f;
      a1[j] = (act && i1 < n && j < n) ? qg.D[((size_t)tt * n + i1) * n + j] : 0.f;
      acc0[j] = 0.f;
      acc1[j] = 0.f;
    }
    if (i0 < n) a0[i0] += sigma;
    if (i1 < n) a1[i1] += sigma;
    auto gram = [&](const float* A, int rows) {  // acc_i += sum_k A[k][i] A[k][:]
      for (int k = 0; k < rows; ++k) {
        row16(r, A + k * n);
        const float s0 = i0 < n ? A[k * n + i0] : 0.f;
        const float s1 = i1 < n ? A[k * n + i1] : 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          acc0[j] = fmaf(s0, r[j], acc0[j]);
          acc1[j] = fmaf(s1, r[j], acc1[j]);
        }
      }
    };
    if (act && m > 0) gram(qs.G + tt * m * n, m);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      a0[j] = fmaf(rho, acc0[j], a0[j]);
      a1[j] = fmaf(rho, acc1[j], a1[j]);
      acc0[j] = 0.f;
      acc1[j] = 0.f;
    }
    if (act) {
      if (t == 0) {
        if (n0 > 0) gram(qs.A0, n0);
        if (N > 0) gram(qs.Am, nx);
      } else {
        gram(qs.Ap + (t - 1) * nx * n, nx);
        if (t < N) gram(qs.Am + t * nx * n, nx);
      }
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      a0[j] = (i0 < n && j < n) ? fmaf(rho_f, acc0[j], a0[j]) : 0.f;
      a1[j] = (i1 < n && j < n) ? fmaf(rho_f, acc1[j], a1[j]) : 0.f;
    }
    if (act) {
      float* d0 = th + t * RowsGeo::TBLK + i0 * RowsGeo::TSTR;
      float* d1 = th + t * RowsGeo::TBLK + i1 * RowsGeo::TSTR;
#pragma unroll
      for (int j = 0; j < 16; j += 4) {
        st128(d0 + j, &a0[j]);
        st128(d1 + j, &a1[j]);
      }
    }
  }
  TMPC_PROF(2);
  // ---- Theta^-1 rows by Gauss-Jordan without row exchanges
  {
    float b0[16], b1[16];  // identity part
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      b0[j] = (j == q && q < n) ? 1.f : 0.f;
      b1[j] = (j == q + 8 && q + 8 < n) ? 1.f : 0.f;
    }
    float* piv = sm + L.tslot + (size_t)(act ? t : 0) * 32;  // the stage's pivot row [Theta part | inverse part]
    bool bad = false;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      if (c < n) {  // n is uniform: every thread takes the same branch
        const bool owner = q == (c & 7);
        if (owner && act) {
          float* ra = c < 8 ? a0 : a1;
          float* rb = c < 8 ? b0 : b1;
          const float p = ra[c];
          if (!(fabsf(p) > 0.f) || !isfinite(p)) bad = true;
          const float inv = 1.f / p;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            ra[j] *= inv;
            rb[j] *= inv;
          }
#pragma unroll
          for (int j = 0; j < 16; j += 4) {
            st128(piv + j, &ra[j]);
            st128(piv + 16 + j, &rb[j]);
          }
        }
        __syncwarp();
        if (act) {
          float pr[16], pb[16];
#pragma unroll
          for (int j = 0; j < 16; j += 4) {
            ld128(&pr[j], piv + j);
            ld128(&pb[j], piv + 16 + j);
          }
          if (!(owner && c < 8)) {
            const float f = a0[c];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              a0[j] = fmaf(-f, pr[j], a0[j]);
              b0[j] = fmaf(-f, pb[j], b0[j]);
            }
          }
          if (!(owner && c >= 8)) {
            const float f = a1[c];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              a1[j] = fmaf(-f, pr[j], a1[j]);
              b1[j] = fmaf(-f, pb[j], b1[j]);
            }
          }
        }
        __syncwarp();
      }
    }
    if (bad) atomicOr(flag, TMPC_STATUS_SINGULAR_BLOCK);
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      save->v[k] = act ? b0[k] : 0.f;
      save->v[16 + k] = act ? b1[k] : 0.f;
    }
  }
  TMPC_PROF(3);
  // ---- Phi rows: S(t, t-1) = Phi_{t-1} rows j, S(t, t+1) = Phi_t^T rows j (columns j of Phi_t)
  {
    float acc0[16], acc1[16], r[16];
    const int j0 = q, j1 = q + 8;
    const bool lo = act && t >= 1;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      acc0[k] = 0.f;
      acc1[k] = 0.f;
    }
    if (lo) {
      const float* ap = qs.Ap + (t - 1) * nx * n;
      const float* am = qs.Am + (t - 1) * nx * n;
      for (int kk = 0; kk < nx; ++kk) {  // acc_j[k] += Ap[kk][j] Am[kk][k]
        row16(r, am + kk * n);
        const float s0 = j0 < n ? ap[kk * n + j0] : 0.f;
        const float s1 = j1 < n ? ap[kk * n + j1] : 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          acc0[k] = fmaf(s0, r[k], acc0[k]);
          acc1[k] = fmaf(s1, r[k], acc1[k]);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const bool in = lo && k < n;
      save->v[32 + k] = (in && j0 < n) ? qg.E[((size_t)(t - 1) * n + j0) * n + k] + rho_f * acc0[k] : 0.f;
      save->v[48 + k] = (in && j1 < n) ? qg.E[((size_t)(t - 1) * n + j1) * n + k] + rho_f * acc1[k] : 0.f;
      acc0[k] = 0.f;
      acc1[k] = 0.f;
    }
    const bool up = act && t < N;
    if (up) {
      const float* ap = qs.Ap + t * nx * n;
      const float* am = qs.Am + t * nx * n;
      for (int kk = 0; kk < nx; ++kk) {  // acc_j[k] += Ap[kk][k] Am[kk][j]
        row16(r, ap + kk * n);
        const float s0 = j0 < n ? am[kk * n + j0] : 0.f;
        const float s1 = j1 < n ? am[kk * n + j1] : 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          acc0[k] = fmaf(r[k], s0, acc0[k]);
          acc1[k] = fmaf(r[k], s1, acc1[k]);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const bool in = up && k < n;
      save->v[64 + k] = (in && j0 < n) ? qg.E[((size_t)t * n + k) * n + j0] + rho_f * acc0[k] : 0.f;
      save->v[80 + k] = (in && j1 < n) ? qg.E[((size_t)t * n + k) * n + j1] + rho_f * acc1[k] : 0.f;
    }
  }
  __syncthreads();
  TMPC_PROF(4);
}

// ADMM-level step 1 (per entry (t, j) of the block vectors): the pending
// over-relaxation of the previous iteration's PCG result (x = alpha x + (1 -
// alpha) x_old, admm.py:893) when `relax`, then x_old = x and
//   gamma = sigma x - q + C^T(rho_f c - y_f) + G^T(rho z - y_g)
// with the targets rho_f c - y_f, rho z - y_g formed inline (the same
// operations and rounding as admm_targets + compute_gamma, without their
// buffers and barrier).  Caller syncs after.
__device__ __forceinline__ void rows_relax_gamma(float* xs, float* xold, float* gam, const QPView<float>& qp,
                                                 const float* yf0, const float* yfd, const float* zg,
                                                 const float* yg, float rho, float rho_f, float sigma, float al,
                                                 bool relax, int T, int n, int nx, int n0, int m) {
  const int N = T - 1;
  TMPC_FOR_ENTRIES(e, o, T, 16, RowsGeo::VSTR) {
    const int t = e >> 4, j = e & 15;
    float xv = xs[o];
    if (relax) {
      xv = al * xv + (1.f - al) * xold[o];
      xs[o] = xv;
    }
    xold[o] = xv;
    float val = 0.f;
    if (j < n) {
      val = sigma * xv - qp.q[t * n + j];
      float eq = 0.f;
      if (t == 0) {
#pragma unroll 4
        for (int k = 0; k < n0; ++k) eq += qp.A0[k * n + j] * (rho_f * qp.c0[k] - yf0[k]);
        if (N > 0) {
#pragma unroll 4
          for (int k = 0; k < nx; ++k) eq += qp.Am[k * n + j] * (rho_f * qp.c[k] - yfd[k]);
        }
      } else {
        const float* ap = qp.Ap + (t - 1) * nx * n;
        const int r0 = (t - 1) * nx;
#pragma unroll 4
        for (int k = 0; k < nx; ++k) eq += ap[k * n + j] * (rho_f * qp.c[r0 + k] - yfd[r0 + k]);
        if (t < N) {
          const float* am = qp.Am + t * nx * n;
          const int r1 = t * nx;
#pragma unroll 4
          for (int k = 0; k < nx; ++k) eq += am[k * n + j] * (rho_f * qp.c[r1 + k] - yfd[r1 + k]);
        }
      }
      val += eq;
      float iq = 0.f;
#pragma unroll 4
      for (int k = 0; k < m; ++k) iq += qp.G[(t * m + k) * n + j] * (rho * zg[t * m + k] - yg[t * m + k]);
      val += iq;
    }
    gam[o] = val;
  }
}

// ADMM-level step 2 (per constraint row): the row of C x / G x on the PCG
// result (before relaxation, admm.py:884-887), then that row's dual update
// and, for inequality rows, the slack / projection update (admm.py:896-931):
// apply_constraints and admm_relax_duals fused row by row (same operations,
// no cx / gx buffers).  The x relaxation is applied by the next step 1 (or
// rows_relax).  Caller syncs after.
__device__ __forceinline__ void rows_constraints_duals(const float* xs, const QPView<float>& qp, float* yf0,
                                                       float* yfd, float* zg, float* yg, float* xig, float rho,
                                                       float rho_f, float al, float sw, bool use_slack, int T,
                                                       int n, int nx, int n0, int m) {
  const int N = T - 1;
  const int tot = n0 + N * nx + T * m;
  for (int e = threadIdx.x; e < tot; e += blockDim.x) {
    if (e < n0) {
      const float cx0 = row_dot(qp.A0 + e * n, xs, n);
      yf0[e] += rho_f * al * (cx0 - qp.c0[e]);
    } else if (e < n0 + N * nx) {
      const int k = e - n0, t = k / nx, i = k - t * nx;
      const float cx = row_dot(qp.Am + (t * nx + i) * n, xs + t * RowsGeo::VSTR, n) +
                       row_dot(qp.Ap + (t * nx + i) * n, xs + (t + 1) * RowsGeo::VSTR, n);
      yfd[k] += rho_f * al * (cx - qp.c[k]);
    } else {
      const int k = e - n0 - N * nx, t = k / m, i = k - t * m;
      const float gx = row_dot(qp.G + (t * m + i) * n, xs + t * RowsGeo::VSTR, n);
      const float zold = zg[k];
      const float zt = al * gx + (1.f - al) * zold + yg[k] / rho;
      float cl = zt;
      const float lb = qp.l[k], ub = qp.u[k];
      if (cl < lb) cl = lb;
      if (cl > ub) cl = ub;
      float znew;
      if (use_slack) {
        const float f = sw / (sw + rho);
        znew = (1.f - f) * zt + f * cl;
        xig[k] = (rho / (sw + rho)) * (cl - zt);
      } else {
        znew = cl;
      }
      zg[k] = znew;
      yg[k] += rho * (al * gx + (1.f - al) * zold - znew);
    }
  }
}

// The pending over-relaxation alone (before a residual check and at exit).
__device__ __forceinline__ void rows_relax(float* xs, const float* xold, float al, int T) {
  TMPC_FOR_ENTRIES(e, o, T, 16, RowsGeo::VSTR) { xs[o] = al * xs[o] + (1.f - al) * xold[o]; }
}

// Staged QP view rebuilt at each use from the offsets in shared memory (kept
// out of registers across the PCG loop).
__device__ __forceinline__ QPView<float> rows_qp_view(float* sm, const RowsSmem& L, const TmpcQP& g, int b, int T,
                                                      int n, int nx, int n0, int m) {
  QPView<float> v = qp_view<float>(g, b, T, n, nx, n0, m);
  v.q = sm + L.sq;
  v.A0 = n0 > 0 ? sm + L.sa0 : nullptr;
  v.Am = sm + L.sam;
  v.Ap = sm + L.sap;
  v.G = m > 0 ? sm + L.sg : nullptr;
  v.c0 = (n0 > 0 && g.c0) ? sm + L.sc0 : nullptr;
  v.c = g.c ? sm + L.sc : nullptr;
  v.l = (m > 0 && g.l) ? sm + L.sl : nullptr;
  v.u = (m > 0 && g.u) ? sm + L.su : nullptr;
  return v;
}

// Register budget: the operator rows (96 registers) are live inside the PCG
// loop only; state that lives across the loop is kept in shared memory (arena
// offsets) or re-read from the kernel parameters.
template <int TM>
__global__ void __launch_bounds__(RowsGeo::TPB * TM, 1) admm_rows_kernel(const AdmmParams<float> P) {
  using R = float;
  constexpr int NB = 16;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  R* sm = reinterpret_cast<R*>(smem_raw);
  __shared__ RowsSmem Ls;
  __shared__ int flag;
  const int b = blockIdx.x;
  if (b >= P.Nb) return;
  TMPC_PROF_INIT
#define TMPC_RS(f) (sm + Ls.f)
  if (threadIdx.x == 0) {
    Ls = RowsSmem(P.T, P.n, P.nx, P.n0, P.m, rows_buf(TM));
    flag = 0;
  }
  __syncthreads();
  {
    const int T = P.T, N = T - 1, n = P.n, nx = P.nx, n0 = P.n0, m = P.m;
    // ---- zero Theta (incl. the padding blocks) and every vector region; load the warm start
    for (size_t e = threadIdx.x; e < (size_t)rows_tpad(T) * RowsGeo::TBLK; e += blockDim.x) TMPC_RS(th)[e] = R(0);
    for (size_t e = Ls.bb + threadIdx.x; e < Ls.yf0; e += blockDim.x) sm[e] = R(0);
    for (int e = threadIdx.x; e < 32; e += blockDim.x) TMPC_RS(red)[kRedSlots + e] = R(0);
    __syncthreads();
    const R* x_in = static_cast<const R*>(P.in.x) + (size_t)b * T * n;
    for (int e = threadIdx.x; e < T * n; e += blockDim.x) {
      const int t = e / n, j = e - t * n;
      TMPC_RS(x)[t * RowsGeo::VSTR + j] = x_in[e];
    }
    if (n0 > 0) {
      const R* a = static_cast<const R*>(P.in.y_f0) + (size_t)b * n0;
      for (int e = threadIdx.x; e < n0; e += blockDim.x) TMPC_RS(yf0)[e] = a[e];
    }
    const R* a = static_cast<const R*>(P.in.y_fdyn) + (size_t)b * N * nx;
    for (int e = threadIdx.x; e < N * nx; e += blockDim.x) TMPC_RS(yfd)[e] = a[e];
    if (m > 0) {
      const R* z = static_cast<const R*>(P.in.z_g) + (size_t)b * T * m;
      const R* y = static_cast<const R*>(P.in.y_g) + (size_t)b * T * m;
      const R* xi = static_cast<const R*>(P.in.xi_g) + (size_t)b * T * m;
      for (int e = threadIdx.x; e < T * m; e += blockDim.x) {
        TMPC_RS(zg)[e] = z[e];
        TMPC_RS(yg)[e] = y[e];
        TMPC_RS(xig)[e] = xi[e];
      }
    }
  }
  R rho = static_cast<const R*>(P.in.rho_bar)[b];

  // The QP copy into the stage area (once), then the operator build; the
  // build is repeated when rho changes.  Both end with a barrier.
  RowOpsSave ops;
  __syncthreads();
  TMPC_PROF(0);
  {
    const QPView<R> qg = qp_view<R>(P.qp, b, P.T, P.n, P.nx, P.n0, P.m);
    rows_stage_qp(sm, Ls, qg, P.T, P.n, P.nx, P.n0, P.m);
    __syncthreads();
  }
  TMPC_PROF(1);
  auto build_operators = [&](R rho_now) {
    const int T = P.T, n = P.n, nx = P.nx, n0 = P.n0, m = P.m;
    const QPView<R> qg = qp_view<R>(P.qp, b, T, n, nx, n0, m);
    const QPView<R> qs = rows_qp_view(sm, Ls, P.qp, b, T, n, nx, n0, m);
    rows_build(sm, &Ls, qg, qs, rho_now * P.rho_f_factor, rho_now, P.sigma, T, n, nx, n0, m, &flag, &ops);
  };
  build_operators(rho);
  TMPC_PROF(5);  // (phases 2-4 timed inside the build; this is the call overhead)

  uint32_t iters = (uint32_t)P.max_iter;
  bool pending = false;  // xs holds a PCG result whose over-relaxation is still to be applied
  for (int it = 0; it < P.max_iter; ++it) {
    const int T = P.T, n = P.n, nx = P.nx, n0 = P.n0, m = P.m;
    const R rho_f = rho * P.rho_f_factor;
    {
      const QPView<R> qp = rows_qp_view(sm, Ls, P.qp, b, T, n, nx, n0, m);
      rows_relax_gamma(TMPC_RS(x), TMPC_RS(xold), TMPC_RS(gam), qp, TMPC_RS(yf0), TMPC_RS(yfd), TMPC_RS(zg),
                       TMPC_RS(yg), rho, rho_f, P.sigma, P.alpha, pending, T, n, nx, n0, m);
      __syncthreads();
    }
    TMPC_PROF(6);
    rows_pcg_cg<rows_buf(TM)>(ops, TMPC_RS(th), TMPC_RS(bb), TMPC_RS(x), TMPC_RS(gam), P.T, P.pcg_max_iter, P.pcg_eps,
                TMPC_RS(red) + kRedSlots);
    pending = true;
    TMPC_PROF(7);
    {
      const QPView<R> qp = rows_qp_view(sm, Ls, P.qp, b, T, n, nx, n0, m);
      const R sw = P.slack_weight ? P.slack_weight[b] : R(0);
      rows_constraints_duals(TMPC_RS(x), qp, TMPC_RS(yf0), TMPC_RS(yfd), TMPC_RS(zg), TMPC_RS(yg), TMPC_RS(xig),
                             rho, rho_f, P.alpha, sw, P.use_slack != 0, T, n, nx, n0, m);
      __syncthreads();
    }
    TMPC_PROF(8);
    if (P.check_every > 0 && (it % P.check_every) == 0) {
      rows_relax(TMPC_RS(x), TMPC_RS(xold), P.alpha, T);
      pending = false;
      __syncthreads();
      const QPView<R> qp = rows_qp_view(sm, Ls, P.qp, b, T, n, nx, n0, m);
      const R sw = P.slack_weight ? P.slack_weight[b] : R(0);
      R rho_new;
      const int st = admm_check<NB>(TMPC_RS(red) + kRedSc, TMPC_RS(red), TMPC_RS(x), TMPC_RS(zg), TMPC_RS(yg),
                                    TMPC_RS(xig), TMPC_RS(yf0), TMPC_RS(yfd), qp, sw, P, it, rho, &rho_new, T, n, nx,
                                    n0, m);
      if (st == 1) {
        iters = (uint32_t)(it + 1);
        break;
      }
      if (st == 2) {
        rho = rho_new;
        build_operators(rho);
      }
      __syncthreads();
    }
  }
  if (pending) {
    rows_relax(TMPC_RS(x), TMPC_RS(xold), P.alpha, P.T);
    __syncthreads();
  }
  TMPC_PROF(9);

  // ---- store
  TMPC_PROF(10);
  bool nonfinite = false;
  {
    const int T = P.T, N = T - 1, n = P.n, nx = P.nx, n0 = P.n0, m = P.m;
    R* xo = static_cast<R*>(P.out.x) + (size_t)b * T * n;
    R* xo2 = P.x_out ? P.x_out + (size_t)b * T * n : nullptr;
    for (int e = threadIdx.x; e < T * n; e += blockDim.x) {
      const int t = e / n, j = e - t * n;
      const R v = TMPC_RS(x)[t * RowsGeo::VSTR + j];
      if (!isfinite(v)) nonfinite = true;
      xo[e] = v;
      if (xo2) xo2[e] = v;
    }
    if (n0 > 0) {
      R* a = static_cast<R*>(P.out.y_f0) + (size_t)b * n0;
      for (int e = threadIdx.x; e < n0; e += blockDim.x) a[e] = TMPC_RS(yf0)[e];
    }
    R* a = static_cast<R*>(P.out.y_fdyn) + (size_t)b * N * nx;
    for (int e = threadIdx.x; e < N * nx; e += blockDim.x) a[e] = TMPC_RS(yfd)[e];
    if (m > 0) {
      R* z = static_cast<R*>(P.out.z_g) + (size_t)b * T * m;
      R* y = static_cast<R*>(P.out.y_g) + (size_t)b * T * m;
      R* xi = static_cast<R*>(P.out.xi_g) + (size_t)b * T * m;
      for (int e = threadIdx.x; e < T * m; e += blockDim.x) {
        z[e] = TMPC_RS(zg)[e];
        y[e] = TMPC_RS(yg)[e];
        xi[e] = TMPC_RS(xig)[e];
      }
    }
  }
#undef TMPC_RS
  if (nonfinite) atomicOr(&flag, TMPC_STATUS_NONFINITE);
  __syncthreads();
  TMPC_PROF(11);
  if (threadIdx.x == 0) {
    static_cast<R*>(P.out.rho_bar)[b] = rho;
    if (P.iters_out) P.iters_out[b] = iters;
    if (P.status_out) P.status_out[b] = flag;
  }
}

inline size_t admm_rows_smem_bytes(int T, int n, int nx, int n0, int m) {
  return RowsSmem(T, n, nx, n0, m, rows_buf(rows_cap(T))).nelem * sizeof(float);
}

// True when the register-resident kernel handles these dimensions.
inline bool admm_rows_applicable(int T, int n, int nx, int n0, int m) {
  return n > 8 && n <= 16 && T >= 2 && T <= RowsGeo::TMAX &&
         (long)admm_rows_smem_bytes(T, n, nx, n0, m) <= max_dyn_smem();
}

}  // namespace tmpc
