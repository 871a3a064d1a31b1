// HBM-streaming PCG on block-tridiagonal operators too large for one CTA's
// shared memory (the linear-system sweep's large T * n corner), and the
// assembly of its operator layout.
//
// Stream layout (per problem, per operator M in {S, Phiinv}):
//     T full NB x NB diagonal blocks D_t, then N full NB x NB sub-diagonal
//     blocks L_t = M(t+1, t), all row-major; S first, then Phiinv.
// Full (not packed) diagonal blocks: every block is read with the same
// coalesced pattern, and the bytes per PCG iteration equal the streaming model
// B_pcg = 2 (2T - 1) n^2 w for n = NB.
//
// Matvec y = M v, one group of G lanes (G = 16 for NB <= 16, else 32) per
// stage t, lane c owning row c of the stage:
//   * lane c loads column c of D_t and of L_t: for every k the group reads
//     row k of the block, so each load instruction is a contiguous
//     NB-element segment (coalesced);
//   * (D_t v_t)[c] and (L_t^T v_{t+1})[c] are lane-local dots (D_t symmetric);
//   * (L_t v_t)[k] = sum_c L_t[k][c] v_t[c] is a sum over the group's lanes:
//     a recursive-halving reduce-scatter leaves row k's total in lane k, which
//     writes it to the `lo` buffer of stage t + 1;
//   * after a barrier y_t = (D_t v_t + L_t^T v_{t+1}) + lo_t.
// The column values of both blocks (2 NB per lane) are loaded before any is
// used, so a warp has 2 NB^2 w bytes in flight; several warps and CTAs per
// SM cover the HBM latency.  Vectors r, p, z (in the y buffer) and lo live in
// shared memory; x is updated in place in the output array.
//
// PCG recurrences and stopping rule: those of pcg_core.cuh (the fused
// reference kernel's, turbompc/solvers/admm/csrc/admm_fused.cu:54-161).
#include "assemble.cuh"
#include "tmpc_common.cuh"

namespace tmpc {

template <int NB, typename R>
struct StreamAcc {
  R* opS;
  R* opP;
  int T;
  static constexpr int B2 = NB * NB;
  __device__ R* sd(int t) const { return opS + (size_t)t * B2; }
  __device__ R* so(int t) const { return opS + (size_t)T * B2 + (size_t)t * B2; }
  __device__ R* pd(int t) const { return opP + (size_t)t * B2; }
  __device__ R* po(int t) const { return opP + (size_t)T * B2 + (size_t)t * B2; }
  __device__ void set_theta(int t, int i, int j, R v) const {
    sd(t)[i * NB + j] = v;
    sd(t)[j * NB + i] = v;
  }
  __device__ R get_theta(int t, int i, int j) const { return sd(t)[i * NB + j]; }
  __device__ void set_phi(int t, int i, int j, R v) const { so(t)[i * NB + j] = v; }
  __device__ R get_phi(int t, int i, int j) const { return so(t)[i * NB + j]; }
  __device__ void set_ntinv(int t, int i, int j, R v) const {
    pd(t)[i * NB + j] = v;
    pd(t)[j * NB + i] = v;
  }
  __device__ R get_ntinv(int t, int i, int j) const { return pd(t)[i * NB + j]; }
  __device__ void set_m(int t, int i, int j, R v) const { po(t)[i * NB + j] = v; }
  __device__ void init() const {}  // every entry (padding included) is written by the assembly
};

template <int NB>
__host__ __device__ constexpr size_t stream_op_elems(int T) {
  return (size_t)(2 * T - 1) * NB * NB;
}

template <int NB, typename R>
__global__ void __launch_bounds__(256) assemble_stream_kernel(TmpcQP qpa, const R* rho, R sigma, R rho_f_factor,
                                                              R* ops, int32_t* status, int Nb, int T, int n, int nx,
                                                              int n0, int m) {
  const int b = blockIdx.x;
  if (b >= Nb) return;
  __shared__ int flag;
  if (threadIdx.x == 0) flag = 0;
  __syncthreads();
  const size_t opn = stream_op_elems<NB>(T);
  const StreamAcc<NB, R> acc{ops + (size_t)b * 2 * opn, ops + (size_t)b * 2 * opn + opn, T};
  const QPView<R> qp = qp_view<R>(qpa, b, T, n, nx, n0, m);
  const R r = rho[b];
  assemble_ops<NB>(acc, qp, r * rho_f_factor, r, sigma, T, n, nx, n0, m, &flag);
  if (threadIdx.x == 0 && status) status[b] = flag;
}

constexpr int kStreamThreads = 256;


// Per-warp staging buffer size (elements): 2 slots x stages per pass x {D, L}.
template <int NB, int G>
__host__ __device__ constexpr int stream_wbuf_elems() {
  return 2 * (32 / G) * 2 * NB * NB;
}

// Lane-local part of one stage: column c of D_t and L_t in dcol / lcol.
template <int NB, typename R, int G>
__device__ __forceinline__ void stream_stage(const R (&dcol)[NB], const R (&lcol)[NB], const R* v, R* y, R* lo,
                                             int t, int c, bool valid, bool hasL) {
  const bool act = c < NB;
  const R* vt = v + (size_t)(valid ? t : 0) * NB;
  const R* vn = v + (size_t)(hasL ? t + 1 : 0) * NB;
  R acc = R(0), accT = R(0);
#pragma unroll
  for (int k = 0; k < NB; ++k) {
    acc = fma(dcol[k], vt[k], acc);
    accT = fma(lcol[k], hasL ? vn[k] : R(0), accT);
  }
  // (L_t v_t)[k] = sum over the group's lanes c of L[k][c] v_t[c].
  const R vc = act ? vt[c] : R(0);
  R part[G];
#pragma unroll
  for (int k = 0; k < G; ++k) part[k] = k < NB ? lcol[k] * vc : R(0);
  // Recursive halving inside the group: after the step with offset o a lane
  // keeps the half of the current index range selected by its bit o.
#pragma unroll
  for (int o = G / 2, len = G / 2; o > 0; o >>= 1, len >>= 1) {
    const bool up = (c & o) != 0;
#pragma unroll
    for (int i = 0; i < len; ++i) {
      const R send = up ? part[i] : part[i + len];
      const R keep = up ? part[i + len] : part[i];
      part[i] = keep + __shfl_xor_sync(0xffffffffu, send, o, 32);
    }
  }
  if (valid && act) {
    y[(size_t)t * NB + c] = acc + accT;
    if (hasL) lo[(size_t)(t + 1) * NB + c] = part[0];
  }
}

// One matvec y_pre = (D v + L^T v_next), lo = L v (shifted one stage); the
// caller syncs and adds lo.  v, y, lo: [T][NB] on chip (lo[0] stays zero).
// STAGE: each warp double-buffers its next pass's blocks in shared memory
// with cp.async (16-byte copies, no registers held), so a warp always has a
// whole pass of blocks in flight; otherwise the columns are loaded straight
// into registers.
template <int NB, typename R, int G, bool STAGE>
__device__ __forceinline__ void stream_matvec(const R* __restrict__ op, int T, const R* v, R* y, R* lo, R* wbuf) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int sub = lane / G, c = lane % G;  // stage slot in the warp, row / column owned
  constexpr int SPW = 32 / G;              // stages per warp pass
  constexpr int B2 = NB * NB;
  const int nw = blockDim.x >> 5;
  const int N = T - 1;
  const bool act = c < NB;
  if constexpr (!STAGE) {
    for (int t0 = wid * SPW; t0 < T; t0 += nw * SPW) {  // warp-uniform trip count
      const int t = t0 + sub;
      const bool valid = t < T;
      const bool hasL = valid && t < N;
      const R* Dt = op + (size_t)(valid ? t : 0) * B2;
      const R* Lt = op + (size_t)T * B2 + (size_t)(hasL ? t : 0) * B2;
      R dcol[NB], lcol[NB];
#pragma unroll
      for (int k = 0; k < NB; ++k) dcol[k] = (valid && act) ? __ldg(Dt + k * NB + c) : R(0);
#pragma unroll
      for (int k = 0; k < NB; ++k) lcol[k] = (hasL && act) ? __ldg(Lt + k * NB + c) : R(0);
      stream_stage<NB, R, G>(dcol, lcol, v, y, lo, t, c, valid, hasL);
    }
  } else {
    constexpr int VEC = 16 / (int)sizeof(R);
    constexpr int CH = B2 / VEC;  // 16-byte chunks per block
    auto issue = [&](int t0, int slot) {
#pragma unroll
      for (int s2 = 0; s2 < SPW; ++s2) {
        const int t = t0 + s2;
        R* dst = wbuf + (size_t)(slot * SPW + s2) * 2 * B2;
        if (t < T) {
          const R* Dt = op + (size_t)t * B2;
          for (int k = lane; k < CH; k += 32) cp_async16(dst + k * VEC, Dt + k * VEC);
          if (t < N) {
            const R* Lt = op + (size_t)T * B2 + (size_t)t * B2;
            for (int k = lane; k < CH; k += 32) cp_async16(dst + B2 + k * VEC, Lt + k * VEC);
          }
        }
      }
      cp_async_commit();
    };
    int slot = 0;
    const int step = nw * SPW;
    issue(wid * SPW, 0);
    for (int t0 = wid * SPW; t0 < T; t0 += step) {
      if (t0 + step < T) {
        issue(t0 + step, slot ^ 1);
      } else {
        cp_async_commit();  // empty group keeps the wait count uniform
      }
      cp_async_wait<1>();
      __syncwarp();
      const int t = t0 + sub;
      const bool valid = t < T;
      const bool hasL = valid && t < N;
      const R* blk = wbuf + (size_t)(slot * SPW + sub) * 2 * B2;
      R dcol[NB], lcol[NB];
#pragma unroll
      for (int k = 0; k < NB; ++k) dcol[k] = (valid && act) ? blk[k * NB + c] : R(0);
#pragma unroll
      for (int k = 0; k < NB; ++k) lcol[k] = (hasL && act) ? blk[B2 + k * NB + c] : R(0);
      stream_stage<NB, R, G>(dcol, lcol, v, y, lo, t, c, valid, hasL);
      __syncwarp();  // every lane is done with this slot before it is refilled
      slot ^= 1;
    }
    cp_async_wait<0>();
  }
}

template <int NB, typename R>
__device__ __forceinline__ R stream_block_sum(R v, R* slots) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) slots[threadIdx.x >> 5] = v;
  __syncthreads();
  R s = R(0);
  const int nw = blockDim.x >> 5;
  for (int w = 0; w < nw; ++w) s += slots[w];
  return s;
}

template <int NB, typename R, bool STAGE>
__global__ void __launch_bounds__(kStreamThreads) pcg_stream_kernel(const R* __restrict__ ops,
                                                                   const R* __restrict__ rhs,
                                                                   const R* __restrict__ x0, R* x_out,
                                                                   uint32_t* iters_out, R eps, int max_iter, int Nb,
                                                                   int T, int n) {
  constexpr int G = NB <= 16 ? 16 : 32;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  R* sm = reinterpret_cast<R*>(smem_raw);
  const int b = blockIdx.x;
  if (b >= Nb) return;
  const size_t opn = stream_op_elems<NB>(T);
  const R* opS = ops + (size_t)b * 2 * opn;
  const R* opP = opS + opn;
  const int VS = T * NB;
  R* r = sm;
  R* p = sm + VS;
  R* y = sm + 2 * VS;
  R* lo = sm + 3 * VS;
  R* red = sm + 4 * VS;  // 2 x 32 slots
  R* wbuf = red + 64 + (size_t)(threadIdx.x >> 5) * stream_wbuf_elems<NB, G>();  // 16-byte aligned
  const int tot = T * n;
  R* x = x_out + (size_t)b * tot;
  const R* g = rhs + (size_t)b * tot;
  // Padded entries (j >= n) of every vector stay exactly zero.
  for (int e = threadIdx.x; e < 4 * VS; e += blockDim.x) sm[e] = R(0);
  __syncthreads();
  for (int e = threadIdx.x; e < tot; e += blockDim.x) {
    const int t = e / n, j = e - t * n;
    p[t * NB + j] = x0[(size_t)b * tot + e];  // p holds x for the first matvec
    x[e] = x0[(size_t)b * tot + e];
  }
  __syncthreads();
  auto matvec = [&](const R* op, const R* v) {
    stream_matvec<NB, R, G, STAGE>(op, T, v, y, lo, wbuf);
    __syncthreads();
  };
  auto idx = [&](int e) { return (e / n) * NB + (e % n); };
  // r = g - S x
  matvec(opS, p);
  for (int e = threadIdx.x; e < tot; e += blockDim.x) {
    const int o = idx(e);
    r[o] = g[e] - (y[o] + lo[o]);
  }
  __syncthreads();
  // z = Phiinv r (into y), p = z, eta = r.z
  matvec(opP, r);
  R part = R(0);
  for (int e = threadIdx.x; e < tot; e += blockDim.x) {
    const int o = idx(e);
    const R z = y[o] + lo[o];
    p[o] = z;
    part = fma(r[o], z, part);
  }
  R eta = stream_block_sum<NB>(part, red);
  const R eta0 = fabs(eta);
  int it = 0;
  for (; it < max_iter; ++it) {
    if (fabs(eta) < R(1e-12) + eps * eta0) break;
    __syncthreads();  // p complete; reduction slots free
    matvec(opS, p);
    part = R(0);
    for (int e = threadIdx.x; e < tot; e += blockDim.x) {
      const int o = idx(e);
      const R sp = y[o] + lo[o];
      y[o] = sp;
      part = fma(p[o], sp, part);
    }
    R den = stream_block_sum<NB>(part, red + 32);
    if (fabs(den) < R(1e-30)) den = R(1e-30);
    const R alpha = eta / den;
    for (int e = threadIdx.x; e < tot; e += blockDim.x) {
      const int o = idx(e);
      x[e] = fma(alpha, p[o], x[e]);
      r[o] = fma(-alpha, y[o], r[o]);
    }
    __syncthreads();
    matvec(opP, r);
    part = R(0);
    for (int e = threadIdx.x; e < tot; e += blockDim.x) {
      const int o = idx(e);
      const R z = y[o] + lo[o];
      y[o] = z;
      part = fma(r[o], z, part);
    }
    const R eta_new = stream_block_sum<NB>(part, red);
    const R beta = eta_new / eta;
    eta = eta_new;
    for (int e = threadIdx.x; e < tot; e += blockDim.x) {
      const int o = idx(e);
      p[o] = fma(beta, p[o], y[o]);
    }
  }
  if (threadIdx.x == 0) iters_out[b] = (uint32_t)it;
}

template <int NB, typename R>
size_t stream_smem_bytes(int T, bool stage) {
  constexpr int G = NB <= 16 ? 16 : 32;
  // 4 T NB is a multiple of 4 elements, so the staging buffers start 16-byte aligned.
  const size_t wb = stage ? (size_t)(kStreamThreads / 32) * stream_wbuf_elems<NB, G>() : 0;
  return (4 * (size_t)T * NB + 64 + wb) * sizeof(R);
}

template <int NB, typename R>
int launch_pcg_stream(const TmpcDims* d, const R* o, const R* rhs, const R* x0, R* xo, uint32_t* it, R eps,
                      int max_iter, cudaStream_t st) {
  const long smax = max_dyn_smem();
  const size_t s_stage = stream_smem_bytes<NB, R>(d->T, true);
  const bool aligned = (reinterpret_cast<uintptr_t>(o) & 15) == 0;
  // Measured on B200: staging pays for the large blocks (NB >= 24: 93 % of
  // the measured HBM copy bandwidth at n = 32, T = 129, fp32, against 47 %
  // with register loads); for NB <= 16 the register path keeps more CTAs per
  // SM and is faster.
  const bool stage = NB >= 24 && aligned && (long)s_stage <= smax;
  const size_t smem = stage ? s_stage : stream_smem_bytes<NB, R>(d->T, false);
  if ((long)smem > smax) return TMPC_ERR_SMEM;
  auto k = stage ? pcg_stream_kernel<NB, R, true> : pcg_stream_kernel<NB, R, false>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  k<<<d->Nb, kStreamThreads, smem, st>>>(o, rhs, x0, xo, it, eps, max_iter, d->Nb, d->T, d->n);
  return (int)cudaPeekAtLastError();
}

template <typename R>
int pcg_stream(const TmpcDims* d, const R* o, const R* rhs, const R* x0, R* xo, uint32_t* it, double eps,
               int32_t max_iter, cudaStream_t st) {
  int rc = check_dims(d);
  if (rc) return rc;
  if (d->Nb == 0) return TMPC_OK;
  if (!o || !rhs || !x0 || !xo || !it) return TMPC_ERR_NULL_ARG;
  return dispatch_nb(d->n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    return launch_pcg_stream<NB, R>(d, o, rhs, x0, xo, it, (R)eps, max_iter, st);
  });
}

template <typename R>
int assemble_stream(const TmpcDims* d, const TmpcQP* qp, const R* rho, double sigma, double rff, R* ops,
                    int32_t* status, cudaStream_t st) {
  int rc = check_dims(d);
  if (rc) return rc;
  if (d->Nb == 0) return TMPC_OK;
  if (!qp || !rho || !ops) return TMPC_ERR_NULL_ARG;
  return dispatch_nb(d->n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    assemble_stream_kernel<NB, R><<<d->Nb, 256, 0, st>>>(*qp, rho, (R)sigma, (R)rff, ops, status, d->Nb, d->T, d->n,
                                                         d->nx, d->n0, d->m);
    return (int)cudaPeekAtLastError();
  });
}

}  // namespace tmpc

extern "C" {

size_t tmpc_stream_operator_bytes(const TmpcDims* dims, int32_t dtype_bytes) {
  if (tmpc::check_dims(dims) || (dtype_bytes != 4 && dtype_bytes != 8)) return 0;
  size_t out = 0;
  tmpc::dispatch_nb(dims->n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    out = (size_t)dims->Nb * 2 * tmpc::stream_op_elems<NB>(dims->T) * (size_t)dtype_bytes;
    return 0;
  });
  return out;
}

int32_t tmpc_schur_assemble_stream_f32(const TmpcDims* dims, const TmpcQP* qp, const float* rho_bar, double sigma,
                                       double rho_f_factor, float* ops, int32_t* status, tmpc_stream_t stream) {
  return tmpc::assemble_stream<float>(dims, qp, rho_bar, sigma, rho_f_factor, ops, status, (cudaStream_t)stream);
}
int32_t tmpc_schur_assemble_stream_f64(const TmpcDims* dims, const TmpcQP* qp, const double* rho_bar, double sigma,
                                       double rho_f_factor, double* ops, int32_t* status, tmpc_stream_t stream) {
  return tmpc::assemble_stream<double>(dims, qp, rho_bar, sigma, rho_f_factor, ops, status, (cudaStream_t)stream);
}
int32_t tmpc_pcg_solve_stream_f32(const TmpcDims* dims, const float* ops, const float* rhs, const float* x0,
                                  float* x_out, uint32_t* iters_out, double eps, int32_t max_iters,
                                  tmpc_stream_t stream) {
  return tmpc::pcg_stream<float>(dims, ops, rhs, x0, x_out, iters_out, eps, max_iters, (cudaStream_t)stream);
}
int32_t tmpc_pcg_solve_stream_f64(const TmpcDims* dims, const double* ops, const double* rhs, const double* x0,
                                  double* x_out, uint32_t* iters_out, double eps, int32_t max_iters,
                                  tmpc_stream_t stream) {
  return tmpc::pcg_stream<double>(dims, ops, rhs, x0, x_out, iters_out, eps, max_iters, (cudaStream_t)stream);
}

}  // extern "C"
