// Linearised discrete dynamics of the built-in models, batched over
// (problem, stage): the producer of the QP's dynamics rows
// (turbompc/problems/optimal_control_problem.py:1217-1272, explicit schemes).
//
//   F(x, u)    one step of the explicit scheme (Euler, midpoint or RK4,
//              turbompc/dynamics/integrators.py:12-76) of the model's x_dot
//   A_minus_t  = [dF/dx, dF/du] at (x_t, u_t)                  (nx x n)
//   c_t        = -F(x_t, u_t) + A_minus_t [x_t; u_t]
//
// Forward-mode differentiation with one tangent per thread: the G threads of
// a stage (G = 16 or 32 >= n) each carry the seed e_j, so thread j produces
// column j of A_minus_t (coalesced stores) and the value F is computed by
// every thread of the stage.  c_t needs sum_j A_ij z_j: a butterfly sum over
// the stage's lanes.
#include <cuda_runtime.h>
#include <math.h>

#include "tmpc_common.cuh"

namespace tmpc {

template <typename R>
struct Dual {
  R v, d;
};
template <typename R>
__device__ __forceinline__ Dual<R> operator+(Dual<R> a, Dual<R> b) { return {a.v + b.v, a.d + b.d}; }
template <typename R>
__device__ __forceinline__ Dual<R> operator-(Dual<R> a, Dual<R> b) { return {a.v - b.v, a.d - b.d}; }
template <typename R>
__device__ __forceinline__ Dual<R> operator*(Dual<R> a, Dual<R> b) { return {a.v * b.v, a.v * b.d + a.d * b.v}; }
template <typename R>
__device__ __forceinline__ Dual<R> operator/(Dual<R> a, Dual<R> b) {
  const R q = a.v / b.v;
  return {q, (a.d - q * b.d) / b.v};
}
template <typename R>
__device__ __forceinline__ Dual<R> operator*(R s, Dual<R> a) { return {s * a.v, s * a.d}; }
template <typename R>
__device__ __forceinline__ Dual<R> operator+(Dual<R> a, R s) { return {a.v + s, a.d}; }
template <typename R>
__device__ __forceinline__ Dual<R> operator-(Dual<R> a, R s) { return {a.v - s, a.d}; }
// sin and cos of a dual number from one sincos of its value.
__device__ __forceinline__ void sc(float v, float* s, float* c) { sincosf(v, s, c); }
__device__ __forceinline__ void sc(double v, double* s, double* c) { sincos(v, s, c); }
template <typename R>
__device__ __forceinline__ void dsincos(Dual<R> a, Dual<R>& s, Dual<R>& c) {
  R sv, cv;
  sc(a.v, &sv, &cv);
  s = {sv, cv * a.d};
  c = {cv, -sv * a.d};
}

// Quadrotor12Dynamics.state_dot (turbompc_b200/dynamics/quadrotor.py), the
// same expression order.  p = {mass, Jx, Jy, Jz, arm_length, yaw_coefficient}.
template <typename R>
__device__ __forceinline__ Dual<R> dscale(Dual<R> a, R s) { return {a.v * s, a.d * s}; }
// a / b with rb = 1 / b.v computed once by the caller.
template <typename R>
__device__ __forceinline__ Dual<R> ddiv(Dual<R> a, Dual<R> b, R rb) {
  const R q = a.v * rb;
  return {q, (a.d - q * b.d) * rb};
}

// Quadrotor12Dynamics.state_dot (turbompc_b200/dynamics/quadrotor.py), the
// same expression order; divisions by cos(theta) and by the constants are
// multiplications by reciprocals formed once.  p = {mass, Jx, Jy, Jz,
// arm_length, yaw_coefficient}; rp = {1/mass, 1/Jx, 1/Jy, 1/Jz}.
template <typename R>
__device__ __forceinline__ void quad_xdot(Dual<R>* out, const Dual<R>* x, const Dual<R>* u, const R* p, const R* rp) {
  const R Jx = p[1], Jy = p[2], Jz = p[3], L = p[4], k = p[5];
  const Dual<R> phi = x[3], th = x[4], psi = x[5];
  const Dual<R> wx = x[9], wy = x[10], wz = x[11];
  const Dual<R> f1 = u[0], f2 = u[1], f3 = u[2], f4 = u[3];
  Dual<R> sph, cph, sth, cth, sps, cps;
  dsincos(phi, sph, cph);
  dsincos(th, sth, cth);
  dsincos(psi, sps, cps);
  const R rc = R(1) / cth.v;
  const Dual<R> tth = ddiv(sth, cth, rc);
  out[0] = x[6];
  out[1] = x[7];
  out[2] = x[8];
  out[3] = (wx + sph * tth * wy) + cph * tth * wz;
  out[4] = cph * wy - sph * wz;
  out[5] = ddiv(sph * wy + cph * wz, cth, rc);
  const Dual<R> F = dscale(((f1 + f2) + f3) + f4, rp[0]);
  out[6] = (cps * sth * cph + sps * sph) * F;
  out[7] = (sps * sth * cph - cps * sph) * F;
  out[8] = cth * cph * F - R(9.81);
  const Dual<R> tx = L * (f2 - f4);
  const Dual<R> ty = L * (f3 - f1);
  const Dual<R> tz = k * (((f1 - f2) + f3) - f4);
  out[9] = dscale(tx - (Jz - Jy) * wy * wz, rp[1]);
  out[10] = dscale(ty - (Jx - Jz) * wz * wx, rp[2]);
  out[11] = dscale(tz - (Jy - Jx) * wx * wy, rp[3]);
}

// ClohessyWiltshireDynamics.state_dot (turbompc_b200/dynamics/spacecraft.py); p = {mean_motion}.
template <typename R>
__device__ __forceinline__ void cw_xdot(Dual<R>* out, const Dual<R>* x, const Dual<R>* u, const R* p) {
  const R nm = p[0];
  out[0] = x[3];
  out[1] = x[4];
  out[2] = x[5];
  out[3] = (R(3) * nm * nm * x[0] + R(2) * nm * x[4]) + u[0];
  out[4] = R(-2) * nm * x[3] + u[1];
  out[5] = R(-1) * nm * nm * x[2] + u[2];
}

template <typename R, int MODEL>
__device__ __forceinline__ void xdot(Dual<R>* out, const Dual<R>* x, const Dual<R>* u, const R* p, const R* rp) {
  if constexpr (MODEL == TMPC_MODEL_QUADROTOR12) quad_xdot(out, x, u, p, rp);
  else cw_xdot(out, x, u, p);
}

template <int MODEL>
struct ModelDims;
template <>
struct ModelDims<TMPC_MODEL_QUADROTOR12> {
  static constexpr int nx = 12, nu = 4, np = 6;
};
template <>
struct ModelDims<TMPC_MODEL_CLOHESSY_WILTSHIRE> {
  static constexpr int nx = 6, nu = 3, np = 1;
};

// One step of the scheme (turbompc_b200/dynamics/integrators.py order).
template <typename R, int MODEL>
__device__ __forceinline__ void step(Dual<R>* xn, const Dual<R>* x, const Dual<R>* u, const R* p, const R* rp,
                                     int scheme, R dt) {
  constexpr int NX = ModelDims<MODEL>::nx;
  Dual<R> k1[NX], tmp[NX];
  xdot<R, MODEL>(k1, x, u, p, rp);
  if (scheme == TMPC_SCHEME_EULER) {
#pragma unroll
    for (int i = 0; i < NX; ++i) xn[i] = x[i] + dt * k1[i];
    return;
  }
  const R h = R(0.5) * dt;
#pragma unroll
  for (int i = 0; i < NX; ++i) tmp[i] = x[i] + h * k1[i];
  if (scheme == TMPC_SCHEME_MIDPOINT) {
    Dual<R> k2[NX];
    xdot<R, MODEL>(k2, tmp, u, p, rp);
#pragma unroll
    for (int i = 0; i < NX; ++i) xn[i] = x[i] + dt * k2[i];
    return;
  }
  Dual<R> acc[NX], k[NX];
  xdot<R, MODEL>(k, tmp, u, p, rp);  // k2
#pragma unroll
  for (int i = 0; i < NX; ++i) {
    acc[i] = k1[i] + R(2) * k[i];
    tmp[i] = x[i] + h * k[i];
  }
  xdot<R, MODEL>(k, tmp, u, p, rp);  // k3
#pragma unroll
  for (int i = 0; i < NX; ++i) {
    acc[i] = acc[i] + R(2) * k[i];
    tmp[i] = x[i] + dt * k[i];
  }
  xdot<R, MODEL>(k, tmp, u, p, rp);  // k4
  const R sixth = R(1.0 / 6.0);
#pragma unroll
  for (int i = 0; i < NX; ++i) xn[i] = x[i] + dt * (sixth * (acc[i] + k[i]));
}

template <typename R>
struct ModelParams {
  R v[8];
};

template <typename R, int MODEL, int G>
__global__ void __launch_bounds__(256) linearize_kernel(int Nb, int T, const R* __restrict__ states,
                                                        const R* __restrict__ controls, R* __restrict__ Am,
                                                        R* __restrict__ c, int scheme, R dt, const ModelParams<R> pp) {
  constexpr int NX = ModelDims<MODEL>::nx, NU = ModelDims<MODEL>::nu, N_ = NX + NU, NP = ModelDims<MODEL>::np;
  static_assert(N_ <= G, "one lane per direction");
  const int N = T - 1;
  const long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long stage = gid / G;  // (b, t) flattened, t < N
  const int j = (int)(gid % G);
  const bool valid = stage < (long)Nb * N;
  const long b = valid ? stage / N : 0;
  const int t = valid ? (int)(stage % N) : 0;
  R p[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) p[i] = pp.v[i];
  R rp[4];  // reciprocals of the quadrotor's mass and inertias (unused by the other models)
#pragma unroll
  for (int i = 0; i < 4; ++i) rp[i] = (MODEL == TMPC_MODEL_QUADROTOR12 && i < NP) ? R(1) / p[i] : R(0);
  Dual<R> x[NX], u[NU], xn[NX];
  const R* xs = states + ((size_t)b * T + t) * NX;
  const R* us = controls + ((size_t)b * T + t) * NU;
#pragma unroll
  for (int i = 0; i < NX; ++i) x[i] = {valid ? xs[i] : R(0), (i == j) ? R(1) : R(0)};
#pragma unroll
  for (int i = 0; i < NU; ++i) u[i] = {valid ? us[i] : R(0), (NX + i == j) ? R(1) : R(0)};
  step<R, MODEL>(xn, x, u, p, rp, scheme, dt);
  // Column j of A_minus_t, and the lane's share of A_minus_t z.
  R zj = R(0);  // z_j by a select chain (no runtime register-array index)
#pragma unroll
  for (int i = 0; i < NX; ++i) zj = (i == j) ? x[i].v : zj;
#pragma unroll
  for (int i = 0; i < NU; ++i) zj = (NX + i == j) ? u[i].v : zj;
  R s[NX];
#pragma unroll
  for (int i = 0; i < NX; ++i) s[i] = (j < N_) ? xn[i].d * zj : R(0);
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1)
#pragma unroll
    for (int i = 0; i < NX; ++i) s[i] += __shfl_xor_sync(0xffffffffu, s[i], o, G);
  if (valid) {
    R* am = Am + (size_t)stage * NX * N_;
    if (j < N_) {
#pragma unroll
      for (int i = 0; i < NX; ++i) am[i * N_ + j] = xn[i].d;
    }
    if (j < NX) {
      R cj = R(0);
#pragma unroll
      for (int i = 0; i < NX; ++i)
        if (i == j) cj = -xn[i].v + s[i];
      c[(size_t)stage * NX + j] = cj;
    }
  }
}

template <typename R>
int linearize(const TmpcDims* d, int32_t model, int32_t scheme, double dt, const R* states, const R* controls,
              const double* params, int32_t n_params, R* Am, R* c, cudaStream_t st) {
  if (!d) return TMPC_ERR_NULL_ARG;
  if (d->Nb < 0 || d->T < 1) return TMPC_ERR_BAD_DIMS;
  if (scheme != TMPC_SCHEME_EULER && scheme != TMPC_SCHEME_MIDPOINT && scheme != TMPC_SCHEME_RK4)
    return TMPC_ERR_UNSUPPORTED;
  int nx, nu, np;
  if (model == TMPC_MODEL_QUADROTOR12) {
    nx = 12; nu = 4; np = 6;
  } else if (model == TMPC_MODEL_CLOHESSY_WILTSHIRE) {
    nx = 6; nu = 3; np = 1;
  } else {
    return TMPC_ERR_UNSUPPORTED;
  }
  if (d->nx != nx || d->n != nx + nu || n_params != np) return TMPC_ERR_BAD_DIMS;
  const long stages = (long)d->Nb * (d->T - 1);
  if (stages == 0) return TMPC_OK;
  if (!states || !controls || !params || !Am || !c) return TMPC_ERR_NULL_ARG;
  ModelParams<R> pb{};  // host values, passed by value with the launch
  for (int i = 0; i < np; ++i) pb.v[i] = (R)params[i];
  constexpr int G = 16;
  const long threads = stages * G;
  const int blocks = (int)((threads + 255) / 256);
  if (model == TMPC_MODEL_QUADROTOR12)
    linearize_kernel<R, TMPC_MODEL_QUADROTOR12, G><<<blocks, 256, 0, st>>>(d->Nb, d->T, states, controls, Am, c,
                                                                           scheme, (R)dt, pb);
  else
    linearize_kernel<R, TMPC_MODEL_CLOHESSY_WILTSHIRE, G><<<blocks, 256, 0, st>>>(d->Nb, d->T, states, controls, Am,
                                                                                  c, scheme, (R)dt, pb);
  return (int)cudaPeekAtLastError();
}

}  // namespace tmpc

extern "C" {

int32_t tmpc_linearize_dynamics_f32(const TmpcDims* dims, int32_t model, int32_t scheme, double dt,
                                    const float* states, const float* controls, const double* params,
                                    int32_t n_params, float* A_minus, float* c, tmpc_stream_t stream) {
  return tmpc::linearize<float>(dims, model, scheme, dt, states, controls, params, n_params, A_minus, c,
                                (cudaStream_t)stream);
}

int32_t tmpc_linearize_dynamics_f64(const TmpcDims* dims, int32_t model, int32_t scheme, double dt,
                                    const double* states, const double* controls, const double* params,
                                    int32_t n_params, double* A_minus, double* c, tmpc_stream_t stream) {
  return tmpc::linearize<double>(dims, model, scheme, dt, states, controls, params, n_params, A_minus, c,
                                 (cudaStream_t)stream);
}

}  // extern "C"
