// lg_slq.cu — stochastic Lanczos quadrature with the Kraemer adjoint.
//
// Reference (python/gpu_eigsh/...):
//   lanczos_torch_noreortho_batched   funm_torch.py:120-173  -> fwd_spmm_kernel, recur_kernel, normalize_kernel
//   _SLQLogdetBatched.forward         funm_torch.py:583-615  -> small_side_kernel (mode 0)
//   _SLQLogdetBatched.backward        funm_torch.py:617-727  -> small_side_kernel gradients, lam_kernel,
//                                                               bwd_spmm_kernel, xi_kernel
//   _small_side / funm_apply_kraemer  funm_torch.py:62-76, 254-373 -> small_side_kernel (modes 1, 2)
//   IMGP precision matvec             imgp.py:192-207, 234-289 -> fwd_spmm_kernel chain (lg_slq_apply),
//                                                               bwd_spmm_kernel chain (lg_slq_apply_vjp)
//
// Operator: A = shift I + L, L = diag(d) + off-diagonal CSR (both directions
// of every edge), applied `power` = nu times: P = A^nu.  The intermediate
// powers A^p v_j (p = 1 .. nu-1) of every Lanczos step are stored for the
// backward pass.
//
// Forward step j, nu >= 2 (nu kernels; h = floor(nu/2)):
//   product 1     v_j = r / ||r|| (the norm from the previous step's column
//                 sums; written), A v_j
//   product nu-h  also the column sums alpha_j = <A^h v_j, A^(nu-h) v_j>
//                 (= <v_j, P v_j>, since A is symmetric)
//   product nu    also r = P v_j - alpha_j v_j - beta_{j-1} v_{j-1} and ||r||^2
// so the three-term recurrence costs no pass of its own.  nu = 1 uses a
// separate recurrence kernel (alpha needs the finished product).
//
// Backward step j (Kraemer reverse sweep; nu + 1 kernels):
//   lam_kernel    lambda = -xi/b + mu x+ + nu x_j from the column dots that
//                 the previous step's last product produced
//   bwd_spmm      M_{p+1} = A M_p (M_0 = lambda).  The operator's parameter
//                 gradient d<lambda, P x_j>/dq = sum_p <A^(nu-1-p) x_j,
//                 (dA/dq) A^p lambda> needs no per-edge storage: the product
//                 that gathers the rows of M_p also applies dA/dq (values
//                 dL/dq on the same sparsity) and dots it with the stored
//                 A^(nu-1-p) x_j of its own row; dA/dshift = I gives the
//                 shift term.  The last product forms xi_{j-1} = -P lambda +
//                 alpha_j lambda + beta_j l+ - beta_j nu x+ and the three
//                 column dots of step j-1.
#include "lg_slq.cuh"
#include "lg_tridiag.cuh"

#include "../../include/lanczos_b200.h"

#include <cmath>
#include <string>
#include <utility>

namespace lg {
extern thread_local std::string g_last_error;
}

namespace lg {
namespace slq {

static int num_sms() {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : 1;
}

// The largest grid (sizes the partial-row buffers): the forward products and
// the light reductions run kMinCta CTAs per SM; the backward products and the
// streaming kernels, built for 2 CTAs per SM (64 registers), run grid2().
int slq_grid() { return kMinCta * num_sms(); }
static int grid2() { return 2 * num_sms(); }

enum { kDotNone = 0, kDotSelf = 1, kDotVj = 2, kDotBlock = 3 };


// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
template <typename T>
struct FwdArgs {
  Op op;
  const T* off;
  const T* diag;
  int ld, B, j, m;
  const T* X;          // input block: r (Z at j = 0) for the first product, else A^(p-1) v_j
  T* Out;              // output block: A^p v_j, or r for the AXPY product
  T* Vj;               // v_j: written by the first product, read by AXPY / kDotVj
  const T* Vjm1;       // v_{j-1} (AXPY; null at j = 0)
  const T* Dsrc;       // kDotBlock partner: A^h v_j
  const double* cin;   // column sums read: first product ||r||^2, AXPY alpha_j
  ColSum cout;         // column sums written: DOT alpha_j, AXPY ||r||^2
  double* alpha;       // (B, m)
  double* beta;        // (B, m)
  double* znorm;       // (B)
};

template <typename T, int LPR, int NCH, bool FIRST, int DOT, bool AXPY>
__global__ void __launch_bounds__(kT, kMinCta) fwd_spmm_kernel(const FwdArgs<T> a) {
  static_assert(!(FIRST && AXPY), "the first product cannot also close the recurrence");
  using G = RowLanes<T, LPR>;
  constexpr int VEC = G::VEC;
  __shared__ double s_k0[kMaxB], s_k1[kMaxB];
  const G g;
  const int B = a.B, ld = a.ld;
  if (FIRST || AXPY) {
    for (int b = threadIdx.x; b < B; b += kT) {
      const double cv = a.cin[b];
      if (FIRST) {
        const double nb = sqrt(cv);
        s_k0[b] = 1.0 / nb;
        if (blockIdx.x == 0) {
          if (a.j == 0) a.znorm[b] = nb;
          else a.beta[(size_t)b * a.m + a.j - 1] = nb;
        }
      } else {
        s_k0[b] = cv;
        s_k1[b] = (a.j > 0) ? a.beta[(size_t)b * a.m + a.j - 1] : 0.0;
        if (blockIdx.x == 0) a.alpha[(size_t)b * a.m + a.j] = cv;
      }
    }
    __syncthreads();
  }
  T k0[NCH][VEC], k1[NCH][VEC];
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      const int c = g.col0(ch) + v;
      k0[ch][v] = (FIRST || AXPY) && c < B ? (T)s_k0[c] : T(0);
      k1[ch][v] = AXPY && c < B ? (T)s_k1[c] : T(0);
    }
  double acc[1][NCH][VEC] = {};
  for (long long wrow = g.first_warp_row(); wrow < a.op.n; wrow += G::stride()) {
    const long long row = wrow + g.sub;
    const bool valid = row < a.op.n;
    T x[NCH][VEC], y[NCH][VEC], unused[NCH][VEC];
    const T dg = valid ? (T)(a.op.shift + (double)__ldg(a.diag + row)) : T(0);
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c0 = g.col0(ch);
#pragma unroll
      for (int v = 0; v < VEC; ++v) x[ch][v] = T(0);
      if (valid && c0 < B) ldvec<T, VEC>(a.X + row * ld + c0, B - c0, x[ch]);
#pragma unroll
      for (int v = 0; v < VEC; ++v) y[ch][v] = dg * x[ch][v];
    }
    gather_rows<T, LPR, NCH, false>(a.op, a.off, nullptr, a.X, ld, B, valid, row, g, y, unused);
    if (!valid) continue;
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c0 = g.col0(ch);
      if (c0 >= B) continue;
      const int nv = B - c0;
      T o[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) o[v] = y[ch][v];
      if (FIRST) {
        // the product is linear: A (x / ||r||) = (A x) / ||r|| per column
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          x[ch][v] *= k0[ch][v];
          o[v] *= k0[ch][v];
        }
        stvec_t<T, VEC>(a.Vj + row * ld + c0, x[ch], nv);
      }
      if (AXPY) {
        T vj[VEC], vm[VEC];
        ldvec<T, VEC>(a.Vj + row * ld + c0, VEC, vj);
#pragma unroll
        for (int v = 0; v < VEC; ++v) vm[v] = T(0);
        if (a.Vjm1) ldvec<T, VEC>(a.Vjm1 + row * ld + c0, VEC, vm);
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          o[v] = o[v] - k0[ch][v] * vj[v] - k1[ch][v] * vm[v];
          acc[0][ch][v] += (double)o[v] * (double)o[v];
        }
      }
      if (DOT != kDotNone) {
        T pv[VEC];
        if (DOT == kDotVj) {
          if (FIRST) {
#pragma unroll
            for (int v = 0; v < VEC; ++v) pv[v] = x[ch][v];
          } else {
            ldvec<T, VEC>(a.Vj + row * ld + c0, VEC, pv);
          }
        } else if (DOT == kDotBlock) {
          ldvec<T, VEC>(a.Dsrc + row * ld + c0, VEC, pv);
        } else {
#pragma unroll
          for (int v = 0; v < VEC; ++v) pv[v] = o[v];
        }
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[0][ch][v] += (double)pv[v] * (double)o[v];
      }
      stvec_t<T, VEC>(a.Out + row * ld + c0, o, nv);
    }
  }
  if (DOT != kDotNone || AXPY) colsum_finish<1, VEC, NCH, LPR>(acc, B, a.cout);
}

// Column sums of X*Y (Y null: of X*X).
template <typename T, int LPR, int NCH>
__global__ void __launch_bounds__(kT, kMinCta) coldot_kernel(int n, int ld, int B, const T* __restrict__ X,
                                                            const T* __restrict__ Y, ColSum cout) {
  using G = RowLanes<T, LPR>;
  constexpr int VEC = G::VEC;
  const G g;
  double acc[1][NCH][VEC] = {};
  for (long long row = g.first_row(); row < n; row += G::stride()) {
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c0 = g.col0(ch);
      if (c0 >= B) continue;
      T x[VEC], y[VEC];
      ldvec<T, VEC>(X + row * ld + c0, B - c0, x);
      if (Y) {
        ldvec<T, VEC>(Y + row * ld + c0, B - c0, y);
      } else {
#pragma unroll
        for (int v = 0; v < VEC; ++v) y[v] = x[v];
      }
#pragma unroll
      for (int v = 0; v < VEC; ++v) acc[0][ch][v] += (double)x[v] * (double)y[v];
    }
  }
  colsum_finish<1, VEC, NCH, LPR>(acc, B, cout);
}

// r = W - alpha_j v_j - beta_{j-1} v_{j-1} (alpha_j from the column sums,
// stored), ||r||^2 to the column sums.
template <typename T, int LPR, int NCH>
__global__ void __launch_bounds__(kT, kMinCta)
recur_kernel(int n, int ld, int B, int j, int m, const T* __restrict__ W, const T* __restrict__ Vj,
             const T* __restrict__ Vjm1, const double* __restrict__ cin, double* alpha, const double* beta,
             T* __restrict__ R, ColSum cout) {
  using G = RowLanes<T, LPR>;
  constexpr int VEC = G::VEC;
  __shared__ double s_a[kMaxB], s_b[kMaxB];
  const G g;
  for (int b = threadIdx.x; b < B; b += kT) {
    s_a[b] = cin[b];
    s_b[b] = (j > 0) ? beta[(size_t)b * m + j - 1] : 0.0;
    if (blockIdx.x == 0) alpha[(size_t)b * m + j] = cin[b];
  }
  __syncthreads();
  T ka[NCH][VEC], kb[NCH][VEC];
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      const int c = g.col0(ch) + v;
      ka[ch][v] = c < B ? (T)s_a[c] : T(0);
      kb[ch][v] = c < B ? (T)s_b[c] : T(0);
    }
  double acc[1][NCH][VEC] = {};
  for (long long row = g.first_row(); row < n; row += G::stride()) {
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c0 = g.col0(ch);
      if (c0 >= B) continue;
      const int nv = B - c0;
      T w[VEC], v[VEC], q[VEC];
      ldvec<T, VEC>(W + row * ld + c0, nv, w);
      ldvec<T, VEC>(Vj + row * ld + c0, nv, v);
#pragma unroll
      for (int i = 0; i < VEC; ++i) q[i] = T(0);
      if (Vjm1) ldvec<T, VEC>(Vjm1 + row * ld + c0, nv, q);
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        w[i] = w[i] - ka[ch][i] * v[i] - kb[ch][i] * q[i];
        acc[0][ch][i] += (double)w[i] * (double)w[i];
      }
      stvec_t<T, VEC>(R + row * ld + c0, w, nv);
    }
  }
  colsum_finish<1, VEC, NCH, LPR>(acc, B, cout);
}

// Vout = R / sqrt(cin) per column; dst[b * dst_stride] = sqrt(cin[b]).
template <typename T, int LPR, int NCH>
__global__ void __launch_bounds__(kT, kMinCta)
normalize_kernel(int n, int ld, int B, const T* __restrict__ R, const double* __restrict__ cin, T* __restrict__ Vout,
                 double* dst, int dst_stride) {
  using G = RowLanes<T, LPR>;
  constexpr int VEC = G::VEC;
  __shared__ double s_s[kMaxB];
  const G g;
  for (int b = threadIdx.x; b < B; b += kT) {
    const double nb = sqrt(cin[b]);
    s_s[b] = 1.0 / nb;
    if (blockIdx.x == 0 && dst) dst[(size_t)b * dst_stride] = nb;
  }
  __syncthreads();
  T ks[NCH][VEC];
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      const int c = g.col0(ch) + v;
      ks[ch][v] = c < B ? (T)s_s[c] : T(0);
    }
  for (long long row = g.first_row(); row < n; row += G::stride()) {
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c0 = g.col0(ch);
      if (c0 >= B) continue;
      T r[VEC];
      ldvec<T, VEC>(R + row * ld + c0, B - c0, r);
#pragma unroll
      for (int i = 0; i < VEC; ++i) r[i] *= ks[ch][i];
      stvec_t<T, VEC>(Vout + row * ld + c0, r, B - c0);
    }
  }
}

// ---------------------------------------------------------------------------
// Small side, one CTA per probe b: T_b = tridiag(alpha[b, :], beta[b, :m-1]),
// T_b = S diag(theta) S^T by bisection + inverse iteration, c = S^T e1.
//   mode 0 (quadratic form): out[b] = ||z_b||^2 sum_i c_i^2 f(theta_i) and its
//          gradient with respect to alpha, beta times g_scale;
//   mode 1 (apply): out[b, :] = f(T_b) e1 = S (f(theta) o c);
//   mode 2 (apply, backward): gradient of <gu[b, :], f(T_b) e1> times g_scale.
// Gradient (Daleckii-Krein): for a scalar <g, f(T) e1>, dT-gradient
// G = S (Gamma o w c^T) S^T with w = S^T g and Gamma the divided differences
// of f at the Ritz values (f' on ties); g_alpha_j = G_jj and
// g_beta_j = G_{j,j+1} + G_{j+1,j}; g_beta[b, m-1] = 0 (the last beta is not
// part of T).  The quadratic form is the case g = ||z||^2 e1.
// ---------------------------------------------------------------------------
__device__ __forceinline__ double fval(int func, double x) {
  switch (func) {
    case LG_FUNC_EXP: return exp(x);
    case LG_FUNC_SQRT: return sqrt(x);
    case LG_FUNC_INV: return 1.0 / x;
    default: return log(x);
  }
}

// (f(xi) - f(xk)) / (xi - xk), written so that it stays accurate as xi -> xk.
__device__ __forceinline__ double fdiv(int func, double xi, double xk, double fi, double fk) {
  const double dl = xi - xk;
  switch (func) {
    case LG_FUNC_EXP: return dl == 0.0 ? fk : fk * (expm1(dl) / dl);
    case LG_FUNC_SQRT: return 1.0 / (fi + fk);
    case LG_FUNC_INV: return -1.0 / (xi * xk);
    default: return dl == 0.0 ? 1.0 / xk : log1p(dl / xk) / dl;
  }
}

__global__ void __launch_bounds__(kQT)
small_side_kernel(int m, int func, int mode, const double* __restrict__ alpha, const double* __restrict__ beta,
                  const double* __restrict__ znorm, const double* __restrict__ gu, double g_scale, double* out,
                  double* g_alpha, double* g_beta, double* scratch, int* status) {
  extern __shared__ double Z[];      // m x m, column-major eigenvectors
  __shared__ double d[kMaxCols], e[kMaxCols], e2[kMaxCols], th[kMaxCols], cf[kMaxCols], fv[kMaxCols],
      wv[kMaxCols];
  __shared__ int cl[kMaxCols];
  __shared__ double sh_nrm, scr[kQT / 32];
  const int b = blockIdx.x, t = threadIdx.x;
  if (t < m) {
    d[t] = alpha[(size_t)b * m + t];
    e[t] = (t < m - 1) ? beta[(size_t)b * m + t] : 0.0;
    e2[t] = e[t] * e[t];
  }
  __syncthreads();
  double* F = scratch + (size_t)b * 4 * kMaxCols * kQT;
  if (!tridiag_eigen_cta<kQT>(d, e, e2, m, th, Z, F, cl, &sh_nrm)) {
    if (t == 0) {
      atomicExch(status, 1);
      if (mode == 0) out[b] = NAN;
    }
    if (t < m) {
      if (mode == 1) {
        out[(size_t)b * m + t] = NAN;
      } else {
        g_alpha[(size_t)b * m + t] = NAN;
        g_beta[(size_t)b * m + t] = NAN;
      }
    }
    return;
  }
  if (t < m) {
    cf[t] = Z[(size_t)t * m];
    fv[t] = fval(func, th[t]);
  }
  __syncthreads();
  if (mode == 1) {
    if (t < m) {
      double s = 0.0;
      for (int i = 0; i < m; ++i) s += Z[t + (size_t)i * m] * (fv[i] * cf[i]);
      out[(size_t)b * m + t] = s;
    }
    return;
  }
  if (mode == 0) {
    const double zz = znorm[b] * znorm[b];
    double part = (t < m) ? cf[t] * cf[t] * fv[t] : 0.0;
    part = block_sum(part, scr);
    if (t == 0) out[b] = zz * part;
    if (t < m) wv[t] = zz * cf[t];
  } else if (t < m) {
    double s = 0.0;
    for (int k = 0; k < m; ++k) s += Z[k + (size_t)t * m] * gu[(size_t)b * m + k];
    wv[t] = s;
  }
  __syncthreads();
  if (t < m) {
    const int j = t;
    const bool has1 = j + 1 < m;
    double ga = 0.0, gb1 = 0.0, gb2 = 0.0;
    for (int i = 0; i < m; ++i) {
      double t1 = 0.0, t2 = 0.0;
      for (int k = 0; k < m; ++k) {
        const double h = fdiv(func, th[i], th[k], fv[i], fv[k]) * cf[k];
        t1 += h * Z[j + (size_t)k * m];
        if (has1) t2 += h * Z[j + 1 + (size_t)k * m];
      }
      const double sw = Z[j + (size_t)i * m] * wv[i];
      ga += sw * t1;
      gb1 += sw * t2;
      if (has1) gb2 += Z[j + 1 + (size_t)i * m] * wv[i] * t1;
    }
    g_alpha[(size_t)b * m + j] = g_scale * ga;
    g_beta[(size_t)b * m + j] = has1 ? g_scale * (gb1 + gb2) : 0.0;
  }
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------
// lambda = -xi/b_j + mu x+ + nu x_j with mu = g*gb_j - <l+, x_j> + <x+, xi>/b_j,
// nu = g*ga_j + <x_j, xi>/b_j (g = *g_out; the three dots come from cin, null
// with xi at j = m-1 where xi = 0).  mu, nu go to munu for the step's last kernel.
template <typename T, int LPR, int NCH>
__global__ void __launch_bounds__(kT, kMinCta)
lam_kernel(int n, int ld, int B, int j, int m, const T* __restrict__ xi, const T* __restrict__ xplus,
           const T* __restrict__ xj, const double* __restrict__ cin, const double* __restrict__ g_alpha,
           const double* __restrict__ g_beta, const double* __restrict__ g_out, const double* __restrict__ beta,
           T* __restrict__ lam, double* munu) {
  using G = RowLanes<T, LPR>;
  constexpr int VEC = G::VEC;
  __shared__ double s_ib[kMaxB], s_mu[kMaxB], s_nu[kMaxB];
  const G g;
  const double gs = g_out ? *g_out : 1.0;
  for (int b = threadIdx.x; b < B; b += kT) {
    const double bj = beta[(size_t)b * m + j];
    const double ib = 1.0 / bj;
    double c1 = 0.0, c2 = 0.0, c3 = 0.0;
    if (cin && xi) {
      c1 = cin[b];
      c2 = cin[kMaxB + b];
      c3 = cin[2 * kMaxB + b];
    }
    s_ib[b] = ib;
    s_mu[b] = gs * g_beta[(size_t)b * m + j] - c1 + c2 * ib;
    s_nu[b] = gs * g_alpha[(size_t)b * m + j] + c3 * ib;
    if (blockIdx.x == 0) {
      munu[b] = s_mu[b];
      munu[kMaxB + b] = s_nu[b];
    }
  }
  __syncthreads();
  T kib[NCH][VEC], kmu[NCH][VEC], knu[NCH][VEC];
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      const int c = g.col0(ch) + v;
      kib[ch][v] = c < B ? (T)s_ib[c] : T(0);
      kmu[ch][v] = c < B ? (T)s_mu[c] : T(0);
      knu[ch][v] = c < B ? (T)s_nu[c] : T(0);
    }
  for (long long row = g.first_row(); row < n; row += G::stride()) {
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c0 = g.col0(ch);
      if (c0 >= B) continue;
      const int nv = B - c0;
      T p[VEC], v[VEC], x[VEC];
      ldvec<T, VEC>(xplus + row * ld + c0, nv, p);
      ldvec<T, VEC>(xj + row * ld + c0, nv, v);
#pragma unroll
      for (int i = 0; i < VEC; ++i) x[i] = T(0);
      if (xi) ldvec<T, VEC>(xi + row * ld + c0, nv, x);
#pragma unroll
      for (int i = 0; i < VEC; ++i) x[i] = -x[i] * kib[ch][i] + kmu[ch][i] * p[i] + knu[ch][i] * v[i];
      stvec_t<T, VEC>(lam + row * ld + c0, x, nv);
    }
  }
}

template <typename T>
struct BwdArgs {
  Op op;
  const T* off;
  const T* doff;
  const T* diag;
  const T* ddiag;
  int ld, B, j, m;
  const T* Min;        // M_p
  const T* Y;          // A^(nu-1-p) x_j
  T* Mout;             // M_{p+1} (not LAST)
  const T* lam;        // LAST: lambda, l+ (null at j = m-1), x+, x_{j-1} (null at j = 0)
  const T* lplus;
  const T* xplus;
  const T* xjm1;
  const double* alpha;
  const double* beta;
  const double* munu;
  T* xi;               // LAST
  ColSum cout;         // LAST with xjm1: <lambda, x_{j-1}>, <x_j, xi>, <x_{j-1}, xi>
  double* sacc;        // per CTA: [2b] += d/dq term, [2b+1] += shift term
};

template <typename T, int LPR, int NCH, bool LAST, bool DERIV>
__global__ void __launch_bounds__(kT, 2) bwd_spmm_kernel(const BwdArgs<T> a) {
  using G = RowLanes<T, LPR>;
  constexpr int VEC = G::VEC;
  __shared__ double s_a[kMaxB], s_b[kMaxB], s_bn[kMaxB], scr[kW];
  const G g;
  const int B = a.B, ld = a.ld;
  if (LAST) {
    for (int b = threadIdx.x; b < B; b += kT) {
      s_a[b] = a.alpha[(size_t)b * a.m + a.j];
      s_b[b] = a.beta[(size_t)b * a.m + a.j];
      s_bn[b] = s_b[b] * a.munu[kMaxB + b];
    }
    __syncthreads();
  }
  const bool dots = LAST && a.xjm1 != nullptr;
  double acc[LAST ? 3 : 1][NCH][VEC] = {};
  double sk = 0.0, sc = 0.0;
  for (long long wrow = g.first_warp_row(); wrow < a.op.n; wrow += G::stride()) {
    const long long row = wrow + g.sub;
    const bool valid = row < a.op.n;
    T mi[NCH][VEC], y[NCH][VEC], yk[NCH][VEC];
    const T dg = valid ? (T)(a.op.shift + (double)__ldg(a.diag + row)) : T(0);
    const T ddg = (DERIV && valid) ? __ldg(a.ddiag + row) : T(0);
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c0 = g.col0(ch);
#pragma unroll
      for (int v = 0; v < VEC; ++v) mi[ch][v] = T(0);
      if (valid && c0 < B) ldvec<T, VEC>(a.Min + row * ld + c0, B - c0, mi[ch]);
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        y[ch][v] = dg * mi[ch][v];
        yk[ch][v] = ddg * mi[ch][v];
      }
    }
    gather_rows<T, LPR, NCH, DERIV>(a.op, a.off, a.doff, a.Min, ld, B, valid, row, g, y, yk);
    if (!valid) continue;
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c0 = g.col0(ch);
      if (c0 >= B) continue;
      const int nv = B - c0;
      T yv[VEC];
      ldvec<T, VEC>(a.Y + row * ld + c0, nv, yv);
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        if (v < nv) {   // yk of a padding column may hold gathered padding values
          if (DERIV) sk += (double)yv[v] * (double)yk[ch][v];
          sc += (double)yv[v] * (double)mi[ch][v];
        }
      }
      if (!LAST) {
        stvec_t<T, VEC>(a.Mout + row * ld + c0, y[ch], nv);
      } else if (dots) {
        // xi_{j-1}; Y is x_j here (p = nu - 1)
        T l[VEC], p[VEC], q[VEC], u[VEC];
        ldvec<T, VEC>(a.lam + row * ld + c0, VEC, l);
        ldvec<T, VEC>(a.xplus + row * ld + c0, VEC, p);
#pragma unroll
        for (int v = 0; v < VEC; ++v) q[v] = T(0);
        if (a.lplus) ldvec<T, VEC>(a.lplus + row * ld + c0, VEC, q);
        ldvec<T, VEC>(a.xjm1 + row * ld + c0, VEC, u);
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          const int c = min(c0 + v, kMaxB - 1);
          const T x = -y[ch][v] + (T)s_a[c] * l[v] + (T)s_b[c] * q[v] - (T)s_bn[c] * p[v];
          y[ch][v] = x;
          acc[0][ch][v] += (double)l[v] * (double)u[v];
          acc[1][ch][v] += (double)yv[v] * (double)x;
          acc[2][ch][v] += (double)u[v] * (double)x;
        }
        stvec_t<T, VEC>(a.xi + row * ld + c0, y[ch], nv);
      }
    }
  }
  const double bsk = DERIV ? block_sum(sk, scr) : 0.0;
  const double bsc = block_sum(sc, scr);
  if (threadIdx.x == 0) {
    a.sacc[2 * blockIdx.x] += bsk;
    a.sacc[2 * blockIdx.x + 1] += bsc;
  }
  if constexpr (LAST) {
    if (dots) colsum_finish<3, VEC, NCH, LPR>(acc, B, a.cout);
  }
}

// Generic reverse step around a caller-formed Plam = P lambda:
// xi = -dcoef (x) G - Plam + alpha_j lam + beta_j l+ - beta_j nu x+ and, with
// x_{j-1}, the three dots of step j-1.  dcoef[b] G[:, b] is the dx term of a
// forward output that depends on the basis directly (funm_apply_kraemer).
template <typename T, int LPR, int NCH>
__global__ void __launch_bounds__(kT, 2)
xi_kernel(int n, int ld, int B, int j, int m, const T* __restrict__ Plam, const T* __restrict__ lam,
          const T* __restrict__ lplus, const T* __restrict__ xplus, const T* __restrict__ xj,
          const T* __restrict__ xjm1, const double* __restrict__ alpha, const double* __restrict__ beta,
          const double* __restrict__ munu, const double* __restrict__ dcoef, const T* __restrict__ Gm,
          T* __restrict__ xi, ColSum cout) {
  using G = RowLanes<T, LPR>;
  constexpr int VEC = G::VEC;
  __shared__ double s_a[kMaxB], s_b[kMaxB], s_bn[kMaxB], s_d[kMaxB];
  const G g;
  for (int b = threadIdx.x; b < B; b += kT) {
    s_a[b] = alpha[(size_t)b * m + j];
    s_b[b] = beta[(size_t)b * m + j];
    s_bn[b] = s_b[b] * munu[kMaxB + b];
    s_d[b] = dcoef ? dcoef[b] : 0.0;
  }
  __syncthreads();
  double acc[3][NCH][VEC] = {};
  for (long long row = g.first_row(); row < n; row += G::stride()) {
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c0 = g.col0(ch);
      if (c0 >= B) continue;
      const int nv = B - c0;
      T w[VEC], l[VEC], p[VEC], q[VEC], gg[VEC];
      ldvec<T, VEC>(Plam + row * ld + c0, nv, w);
      ldvec<T, VEC>(lam + row * ld + c0, nv, l);
      ldvec<T, VEC>(xplus + row * ld + c0, nv, p);
#pragma unroll
      for (int i = 0; i < VEC; ++i) q[i] = gg[i] = T(0);
      if (lplus) ldvec<T, VEC>(lplus + row * ld + c0, nv, q);
      if (Gm) ldvec<T, VEC>(Gm + row * ld + c0, nv, gg);
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const int c = min(c0 + i, kMaxB - 1);
        w[i] = -(T)s_d[c] * gg[i] - w[i] + (T)s_a[c] * l[i] + (T)s_b[c] * q[i] - (T)s_bn[c] * p[i];
      }
      stvec_t<T, VEC>(xi + row * ld + c0, w, nv);
      if (xjm1) {
        T u[VEC], v[VEC];
        ldvec<T, VEC>(xjm1 + row * ld + c0, nv, u);
        ldvec<T, VEC>(xj + row * ld + c0, nv, v);
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          acc[0][ch][i] += (double)l[i] * (double)u[i];
          acc[1][ch][i] += (double)v[i] * (double)w[i];
          acc[2][ch][i] += (double)u[i] * (double)w[i];
        }
      }
    }
  }
  if (xjm1) colsum_finish<3, VEC, NCH, LPR>(acc, B, cout);
}

// gZ = (<xi, v0> v0 - xi) / ||z|| + g_zn * z / ||z||  per column (the gradient
// with respect to the start vector; <xi, v0> from cin).
template <typename T, int LPR, int NCH>
__global__ void __launch_bounds__(kT, kMinCta)
start_grad_kernel(int n, int ld, int B, const T* __restrict__ xi, const T* __restrict__ V0, const T* __restrict__ Z,
                  const double* __restrict__ znorm, const double* __restrict__ g_zn, const double* __restrict__ cin,
                  T* __restrict__ gZ) {
  using G = RowLanes<T, LPR>;
  constexpr int VEC = G::VEC;
  __shared__ double s_d[kMaxB], s_i[kMaxB], s_g[kMaxB];
  const G g;
  for (int b = threadIdx.x; b < B; b += kT) {
    s_d[b] = cin[b];
    s_i[b] = 1.0 / znorm[b];
    s_g[b] = g_zn ? g_zn[b] : 0.0;
  }
  __syncthreads();
  for (long long row = g.first_row(); row < n; row += G::stride()) {
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int c0 = g.col0(ch);
      if (c0 >= B) continue;
      const int nv = B - c0;
      T x[VEC], v[VEC], z[VEC];
      ldvec<T, VEC>(xi + row * ld + c0, nv, x);
      ldvec<T, VEC>(V0 + row * ld + c0, nv, v);
      ldvec<T, VEC>(Z + row * ld + c0, nv, z);
      double r[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const int c = min(c0 + i, kMaxB - 1);
        r[i] = ((s_d[c] * (double)v[i] - (double)x[i]) + s_g[c] * (double)z[i]) * s_i[c];
      }
      stvec<T, VEC>(gZ + row * ld + c0, r, nv);
    }
  }
}

__global__ void sacc_reduce_kernel(const double* __restrict__ sacc, int rows, double* out) {
  __shared__ double s0[32], s1[32];
  const int t = threadIdx.x;
  double a = 0.0, b = 0.0;
  for (int r = t; r < rows; r += 32) {
    a += sacc[2 * r];
    b += sacc[2 * r + 1];
  }
  s0[t] = a;
  s1[t] = b;
  __syncwarp();
  if (t == 0) {
    double x = 0.0, y = 0.0;
    for (int i = 0; i < 32; ++i) {
      x += s0[i];
      y += s1[i];
    }
    out[0] = x;
    out[1] = y;
  }
}

// gA += lam x^T (dense n x n, row-major; B = 1 blocks with row stride ld).
template <typename T>
__global__ void outer_acc_kernel(int n, int ld, const T* __restrict__ lam, const T* __restrict__ x,
                                 double* __restrict__ gA) {
  const long long total = (long long)n * n;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / n, c = i - r * n;
    gA[i] += (double)lam[r * ld] * (double)x[c * ld];
  }
}

// y = A x for a dense row-major n x n A (one warp per row; B = 1 blocks).
template <typename T>
__global__ void __launch_bounds__(kT, kMinCta)
dense_matvec_kernel(int n, const T* __restrict__ A, const T* __restrict__ x, int ldx, T* __restrict__ y, int ldy) {
  const int lane = threadIdx.x & 31;
  for (long long row = (long long)blockIdx.x * kW + (threadIdx.x >> 5); row < n; row += (long long)gridDim.x * kW) {
    double s = 0.0;
    for (int c = lane; c < n; c += 32) s += (double)A[row * n + c] * (double)x[(long long)c * ldx];
    s = warp_sum(s);
    if (lane == 0) y[row * ldy] = (T)s;
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static size_t al256(size_t b) { return (b + 255) / 256 * 256; }

struct Ws {
  ColSum cs[2];
  double* sacc;
  double* munu;
  double* qscr;
  char* blocks;
  size_t vb;
  size_t bytes;
};

static int num_blocks(int power) { return power + 1 > 5 ? power + 1 : 5; }

static size_t ws_layout(int n, int ld, int es, int B, int power, int grid, char* base, Ws* w) {
  size_t o = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? base + o : nullptr;
    o += al256(bytes);
    return p;
  };
  unsigned* ctr = reinterpret_cast<unsigned*>(take(2 * sizeof(unsigned)));
  Ws t;
  for (int k = 0; k < 2; ++k) {
    t.cs[k].part = reinterpret_cast<double*>(take((size_t)grid * kRowStride * sizeof(double)));
    t.cs[k].out = reinterpret_cast<double*>(take((size_t)kRowStride * sizeof(double)));
    t.cs[k].counter = ctr ? ctr + k : nullptr;
  }
  t.sacc = reinterpret_cast<double*>(take((size_t)2 * grid * sizeof(double)));
  t.munu = reinterpret_cast<double*>(take((size_t)2 * kMaxB * sizeof(double)));
  t.qscr = reinterpret_cast<double*>(take((size_t)(B > 0 ? B : 1) * 4 * kMaxCols * kQT * sizeof(double)));
  t.vb = al256((size_t)n * ld * es);
  t.blocks = take(t.vb * (n > 0 ? num_blocks(power) : 0));
  t.bytes = o;
  if (w) *w = t;
  return o;
}

static char* block(const Ws& w, int i) { return w.blocks + w.vb * i; }

static bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

static int fail(const char* what) {
  g_last_error = what;
  return LG_ERR_INVALID;
}

static int cuda_fail(const char* where, cudaError_t e) {
  g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
  return LG_ERR_CUDA;
}

static int check_block(int n, int B, int ld, int dtype) {
  if (n < 1) return fail("lg_slq: n must be >= 1");
  if (B < 1 || B > kMaxB) return fail("lg_slq: B (active columns) must be in [1, 128]");
  if (ld < B || ld % (dtype == LG_F64 ? 2 : 4) != 0)
    return fail("lg_slq: ld must be >= B and a multiple of 4 (fp32) or 2 (fp64)");
  if (dtype != LG_F32 && dtype != LG_F64) return fail("lg_slq: dtype must be LG_F32 or LG_F64");
  return LG_OK;
}

static int check_op(const lg_slq_op* op, int B, int ld) {
  if (!op) return fail("lg_slq: null operator");
  int rc = check_block(op->n, B, ld, op->dtype);
  if (rc != LG_OK) return rc;
  if (op->power < 1 || op->power > 8) return fail("lg_slq: power must be in [1, 8]");
  if (op->nnz < 0 || op->nnz > 2147483647LL) return fail("lg_slq: nnz must be in [0, 2^31)");
  if (!op->rowptr || !op->diag || (op->nnz > 0 && (!op->col || !op->offval)))
    return fail("lg_slq: operator arrays missing");
  if ((op->ddiag && op->nnz > 0 && !op->doffval) || (!op->ddiag && op->doffval))
    return fail("lg_slq: ddiag and doffval go together");
  return LG_OK;
}

static int check_ws(void* ws, size_t ws_bytes, size_t need) {
  if (!ws || !aligned(ws, 256)) return fail("lg_slq: workspace must be a 256-byte aligned device buffer");
  if (ws_bytes < need) return fail("lg_slq: workspace too small (see lg_slq_workspace_bytes)");
  return LG_OK;
}

static int check_ptr(const void* p, int dtype, const char* what) {
  if (!p) {
    g_last_error = std::string("lg_slq: null ") + what;
    return LG_ERR_INVALID;
  }
  if (!aligned(p, dtype == LG_F64 ? 16 : 8)) {
    g_last_error = std::string("lg_slq: misaligned ") + what;
    return LG_ERR_INVALID;
  }
  return LG_OK;
}

static cudaError_t reset_counters(const Ws& w, cudaStream_t st) {
  return cudaMemsetAsync(w.cs[0].counter, 0, 2 * sizeof(unsigned), st);
}

// ---- launch helpers ------------------------------------------------------
template <typename T, int LPR, int NCH>
static void launch_fwd(bool first, int dot, bool axpy, const FwdArgs<T>& a, int grid, cudaStream_t st) {
  if (first) {
    if (dot == kDotSelf) fwd_spmm_kernel<T, LPR, NCH, true, kDotSelf, false><<<grid, kT, 0, st>>>(a);
    else if (dot == kDotVj) fwd_spmm_kernel<T, LPR, NCH, true, kDotVj, false><<<grid, kT, 0, st>>>(a);
    else fwd_spmm_kernel<T, LPR, NCH, true, kDotNone, false><<<grid, kT, 0, st>>>(a);
  } else if (axpy) {
    fwd_spmm_kernel<T, LPR, NCH, false, kDotNone, true><<<grid, kT, 0, st>>>(a);
  } else if (dot == kDotSelf) {
    fwd_spmm_kernel<T, LPR, NCH, false, kDotSelf, false><<<grid, kT, 0, st>>>(a);
  } else if (dot == kDotBlock) {
    fwd_spmm_kernel<T, LPR, NCH, false, kDotBlock, false><<<grid, kT, 0, st>>>(a);
  } else {
    fwd_spmm_kernel<T, LPR, NCH, false, kDotNone, false><<<grid, kT, 0, st>>>(a);
  }
}

template <typename T, int LPR, int NCH>
static void launch_bwd(bool last, bool deriv, const BwdArgs<T>& a, int grid, cudaStream_t st) {
  if (last) {
    if (deriv) bwd_spmm_kernel<T, LPR, NCH, true, true><<<grid2(), kT, 0, st>>>(a);
    else bwd_spmm_kernel<T, LPR, NCH, true, false><<<grid2(), kT, 0, st>>>(a);
  } else {
    if (deriv) bwd_spmm_kernel<T, LPR, NCH, false, true><<<grid2(), kT, 0, st>>>(a);
    else bwd_spmm_kernel<T, LPR, NCH, false, false><<<grid2(), kT, 0, st>>>(a);
  }
}

static Op make_op(const lg_slq_op& o) { return Op{o.n, o.rowptr, o.col, o.shift}; }

// ---- fused forward (recurrence through the sparse products) --------------
template <typename T, int LPR, int NS>
static cudaError_t forward_t(const lg_slq_op& o, int B, int m, int ld, const T* Z, T* V, T* Yst, double* alpha,
                             double* beta, double* znorm, const Ws& w, int grid, cudaStream_t st) {
  const int nu = o.power, h = nu / 2, pdot = nu - h;
  const size_t bs = (size_t)o.n * ld;
  T* R = reinterpret_cast<T*>(block(w, 0));
  T* W = reinterpret_cast<T*>(block(w, 1));
  auto Yp = [&](int j, int p) { return Yst + ((size_t)j * (nu - 1) + (p - 1)) * bs; };   // A^p v_j, p >= 1
  coldot_kernel<T, LPR, NS><<<grid, kT, 0, st>>>(o.n, ld, B, Z, nullptr, w.cs[0]);
  FwdArgs<T> a{};
  a.op = make_op(o);
  a.off = static_cast<const T*>(o.offval);
  a.diag = static_cast<const T*>(o.diag);
  a.ld = ld;
  a.B = B;
  a.m = m;
  a.alpha = alpha;
  a.beta = beta;
  a.znorm = znorm;
  for (int j = 0; j < m; ++j) {
    a.j = j;
    a.Vj = V + (size_t)j * bs;
    a.Vjm1 = j > 0 ? V + (size_t)(j - 1) * bs : nullptr;
    if (nu == 1) {
      a.X = (j == 0) ? Z : R;
      a.Out = W;
      a.cin = w.cs[0].out;
      a.cout = w.cs[1];
      launch_fwd<T, LPR, NS>(true, kDotVj, false, a, grid, st);
      recur_kernel<T, LPR, NS><<<grid, kT, 0, st>>>(o.n, ld, B, j, m, W, a.Vj, a.Vjm1, w.cs[1].out, alpha, beta, R,
                                                w.cs[0]);
      continue;
    }
    for (int p = 1; p <= nu; ++p) {
      const bool first = (p == 1), axpy = (p == nu);
      int dot = kDotNone;
      if (p == pdot) dot = (h == nu - h) ? kDotSelf : kDotBlock;
      a.X = first ? ((j == 0) ? Z : R) : Yp(j, p - 1);
      a.Out = axpy ? R : Yp(j, p);
      a.Dsrc = (dot == kDotBlock) ? Yp(j, h) : nullptr;
      a.cin = first ? w.cs[0].out : (axpy ? w.cs[1].out : nullptr);
      a.cout = axpy ? w.cs[0] : w.cs[1];
      launch_fwd<T, LPR, NS>(first, dot, axpy, a, grid, st);
    }
  }
  normalize_kernel<T, LPR, NS><<<grid, kT, 0, st>>>(o.n, ld, B, R, w.cs[0].out, V + (size_t)m * bs, beta + (m - 1), m);
  return cudaGetLastError();
}

// ---- fused backward --------------------------------------------------------
template <typename T, int LPR, int NS>
static cudaError_t backward_t(const lg_slq_op& o, int B, int m, int ld, const T* V, const T* Yst,
                              const double* alpha, const double* beta, const double* g_alpha, const double* g_beta,
                              const double* g_out, double* g_params, const Ws& w, int grid, cudaStream_t st) {
  const int nu = o.power;
  const size_t bs = (size_t)o.n * ld;
  const bool deriv = o.ddiag != nullptr;
  T* xi = reinterpret_cast<T*>(block(w, 0));
  T* lam = reinterpret_cast<T*>(block(w, 1));
  T* lplus = reinterpret_cast<T*>(block(w, 2));
  T* M[2] = {reinterpret_cast<T*>(block(w, 3)), reinterpret_cast<T*>(block(w, 4))};
  auto Yp = [&](int j, int p) { return Yst + ((size_t)j * (nu - 1) + (p - 1)) * bs; };
  cudaError_t e = cudaMemsetAsync(w.sacc, 0, (size_t)2 * grid * sizeof(double), st);
  if (e != cudaSuccess) return e;
  BwdArgs<T> a{};
  a.op = make_op(o);
  a.off = static_cast<const T*>(o.offval);
  a.doff = static_cast<const T*>(o.doffval);
  a.diag = static_cast<const T*>(o.diag);
  a.ddiag = static_cast<const T*>(o.ddiag);
  a.ld = ld;
  a.B = B;
  a.m = m;
  a.alpha = alpha;
  a.beta = beta;
  a.munu = w.munu;
  a.sacc = w.sacc;
  a.cout = w.cs[1];
  bool have_lplus = false;
  for (int j = m - 1; j >= 0; --j) {
    const T* xj = V + (size_t)j * bs;
    const T* xplus = V + (size_t)(j + 1) * bs;
    const bool top = (j == m - 1);
    lam_kernel<T, LPR, NS><<<grid, kT, 0, st>>>(o.n, ld, B, j, m, top ? nullptr : xi, xplus, xj,
                                            top ? nullptr : w.cs[1].out, g_alpha, g_beta, g_out, beta, lam, w.munu);
    a.j = j;
    a.lam = lam;
    a.lplus = have_lplus ? lplus : nullptr;
    a.xplus = xplus;
    a.xjm1 = (j > 0) ? V + (size_t)(j - 1) * bs : nullptr;
    a.xi = xi;
    const T* Min = lam;
    for (int p = 0; p < nu; ++p) {
      const bool last = (p == nu - 1);
      a.Min = Min;
      a.Y = last ? xj : Yp(j, nu - 1 - p);
      a.Mout = last ? nullptr : M[p & 1];
      launch_bwd<T, LPR, NS>(last, deriv, a, grid, st);
      Min = a.Mout;
    }
    std::swap(lam, lplus);
    have_lplus = true;
  }
  sacc_reduce_kernel<<<1, 32, 0, st>>>(w.sacc, grid, g_params);
  return cudaGetLastError();
}

// ---- operator apply and its VJP -------------------------------------------
template <typename T, int LPR, int NS>
static cudaError_t apply_t(const lg_slq_op& o, int B, int ld, const T* X, T* Yout, const Ws& w, int grid,
                           cudaStream_t st) {
  FwdArgs<T> a{};
  a.op = make_op(o);
  a.off = static_cast<const T*>(o.offval);
  a.diag = static_cast<const T*>(o.diag);
  a.ld = ld;
  a.B = B;
  const T* in = X;
  for (int p = 1; p <= o.power; ++p) {
    a.X = in;
    a.Out = (p == o.power) ? Yout : reinterpret_cast<T*>(block(w, p & 1));
    launch_fwd<T, LPR, NS>(false, kDotNone, false, a, grid, st);
    in = a.Out;
  }
  return cudaGetLastError();
}

template <typename T, int LPR, int NS>
static cudaError_t apply_vjp_t(const lg_slq_op& o, int B, int ld, const T* X, const T* G, T* gX, double* g_params,
                               const Ws& w, int grid, cudaStream_t st) {
  const int nu = o.power;
  // powers X_q = A^q X, q = 1 .. nu-1, in blocks 2 .. nu
  auto Xq = [&](int q) -> T* { return reinterpret_cast<T*>(block(w, 1 + q)); };
  FwdArgs<T> f{};
  f.op = make_op(o);
  f.off = static_cast<const T*>(o.offval);
  f.diag = static_cast<const T*>(o.diag);
  f.ld = ld;
  f.B = B;
  for (int q = 1; q < nu; ++q) {
    f.X = (q == 1) ? X : Xq(q - 1);
    f.Out = Xq(q);
    launch_fwd<T, LPR, NS>(false, kDotNone, false, f, grid, st);
  }
  cudaError_t e = cudaMemsetAsync(w.sacc, 0, (size_t)2 * grid * sizeof(double), st);
  if (e != cudaSuccess) return e;
  BwdArgs<T> a{};
  a.op = f.op;
  a.off = f.off;
  a.doff = static_cast<const T*>(o.doffval);
  a.diag = f.diag;
  a.ddiag = static_cast<const T*>(o.ddiag);
  a.ld = ld;
  a.B = B;
  a.sacc = w.sacc;
  const bool deriv = o.ddiag != nullptr;
  const T* Min = G;
  T* M[2] = {reinterpret_cast<T*>(block(w, 0)), reinterpret_cast<T*>(block(w, 1))};
  for (int p = 0; p < nu; ++p) {
    a.Min = Min;
    a.Y = (p == nu - 1) ? X : Xq(nu - 1 - p);
    a.Mout = (p == nu - 1) ? gX : M[p & 1];
    launch_bwd<T, LPR, NS>(false, deriv, a, grid, st);
    Min = a.Mout;
  }
  sacc_reduce_kernel<<<1, 32, 0, st>>>(w.sacc, grid, g_params);
  return cudaGetLastError();
}

}  // namespace slq
}  // namespace lg

using namespace lg;
using namespace lg::slq;

// Lane layout <T, LPR, NS> of every block kernel by element type and probe
// count (the last argument is unused): the fewest lanes per row that cover the
// row's 16-byte vectors, so that a block of few probes (one shard of the
// probes on one of several GPUs) keeps every lane busy.
#define LG_DISPATCH(DTYPE, B, CALL)                                                                   \
  ((DTYPE) == LG_F64                                                                                   \
       ? ((B) <= 8 ? CALL(double, 4, 1, 1) : (B) <= 16 ? CALL(double, 8, 1, 1)                         \
          : (B) <= 32 ? CALL(double, 16, 1, 1) : (B) <= 64 ? CALL(double, 32, 1, 1) : CALL(double, 32, 2, 2)) \
       : ((B) <= 8 ? CALL(float, 2, 1, 1) : (B) <= 16 ? CALL(float, 4, 1, 1)                            \
          : (B) <= 32 ? CALL(float, 8, 1, 1) : (B) <= 64 ? CALL(float, 16, 1, 1) : CALL(float, 32, 1, 2)))
extern "C" size_t lg_slq_workspace_bytes(const lg_slq_op* op, int B, int ld) {
  if (op) {
    if (check_op(op, B, ld) != LG_OK) return 0;
    return ws_layout(op->n, ld, op->dtype == LG_F64 ? 8 : 4, B, op->power, slq_grid(), nullptr, nullptr);
  }
  if (B < 1 || B > kMaxB) return 0;
  return ws_layout(0, 0, 4, B, 1, slq_grid(), nullptr, nullptr);
}

static int prepare(const lg_slq_op* op, int B, int ld, void* ws, size_t ws_bytes, Ws* w, int* grid) {
  int rc = check_op(op, B, ld);
  if (rc != LG_OK) return rc;
  *grid = slq_grid();
  const int es = op->dtype == LG_F64 ? 8 : 4;
  rc = check_ws(ws, ws_bytes, ws_layout(op->n, ld, es, B, op->power, *grid, nullptr, nullptr));
  if (rc != LG_OK) return rc;
  ws_layout(op->n, ld, es, B, op->power, *grid, static_cast<char*>(ws), w);
  return LG_OK;
}

extern "C" int lg_slq_forward(const lg_slq_op* op, int B, int m, int ld, const void* Z, void* V, void* Y,
                              double* alpha, double* beta, double* znorm, void* ws, size_t ws_bytes, void* stream) {
  Ws w;
  int grid = 0;
  int rc = prepare(op, B, ld, ws, ws_bytes, &w, &grid);
  if (rc != LG_OK) return rc;
  if (m < 1 || m > kMaxCols) return fail("lg_slq_forward: m must be in [1, 128]");
  if ((rc = check_ptr(Z, op->dtype, "Z")) || (rc = check_ptr(V, op->dtype, "V"))) return rc;
  if (op->power > 1 && (rc = check_ptr(Y, op->dtype, "Y"))) return rc;
  if (!alpha || !beta || !znorm) return fail("lg_slq_forward: null alpha/beta/znorm");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = reset_counters(w, st);
  if (e == cudaSuccess) {
#define LG_FWD(TT, L, NS, NP)                                                                                           \
  forward_t<TT, L, NS>(*op, B, m, ld, static_cast<const TT*>(Z), static_cast<TT*>(V), static_cast<TT*>(Y), alpha, beta, \
                   znorm, w, grid, st)
    e = LG_DISPATCH(op->dtype, B, LG_FWD);
#undef LG_FWD
  }
  return e == cudaSuccess ? LG_OK : cuda_fail("lg_slq_forward", e);
}

extern "C" int lg_slq_backward(const lg_slq_op* op, int B, int m, int ld, const void* V, const void* Y,
                               const double* alpha, const double* beta, const double* g_alpha, const double* g_beta,
                               const double* g_out, double* g_params, void* ws, size_t ws_bytes, void* stream) {
  Ws w;
  int grid = 0;
  int rc = prepare(op, B, ld, ws, ws_bytes, &w, &grid);
  if (rc != LG_OK) return rc;
  if (m < 1 || m > kMaxCols) return fail("lg_slq_backward: m must be in [1, 128]");
  if ((rc = check_ptr(V, op->dtype, "V"))) return rc;
  if (op->power > 1 && (rc = check_ptr(Y, op->dtype, "Y"))) return rc;
  if (!alpha || !beta || !g_alpha || !g_beta || !g_params) return fail("lg_slq_backward: null scalar arrays");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = reset_counters(w, st);
  if (e == cudaSuccess) {
#define LG_BWD(TT, L, NS, NP)                                                                                       \
  backward_t<TT, L, NS>(*op, B, m, ld, static_cast<const TT*>(V), static_cast<const TT*>(Y), alpha, beta, g_alpha, \
                    g_beta, g_out, g_params, w, grid, st)
    e = LG_DISPATCH(op->dtype, B, LG_BWD);
#undef LG_BWD
  }
  return e == cudaSuccess ? LG_OK : cuda_fail("lg_slq_backward", e);
}

extern "C" int lg_slq_apply(const lg_slq_op* op, int B, int ld, const void* X, void* Y, void* ws, size_t ws_bytes,
                            void* stream) {
  Ws w;
  int grid = 0;
  int rc = prepare(op, B, ld, ws, ws_bytes, &w, &grid);
  if (rc != LG_OK) return rc;
  if ((rc = check_ptr(X, op->dtype, "X")) || (rc = check_ptr(Y, op->dtype, "Y"))) return rc;
  if (X == Y) return fail("lg_slq_apply: X and Y must not alias");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define LG_APPLY(TT, L, NS, NP) apply_t<TT, L, NS>(*op, B, ld, static_cast<const TT*>(X), static_cast<TT*>(Y), w, grid, st)
  cudaError_t e = LG_DISPATCH(op->dtype, B, LG_APPLY);
#undef LG_APPLY
  return e == cudaSuccess ? LG_OK : cuda_fail("lg_slq_apply", e);
}

extern "C" int lg_slq_apply_vjp(const lg_slq_op* op, int B, int ld, const void* X, const void* G, void* gX,
                                double* g_params, void* ws, size_t ws_bytes, void* stream) {
  Ws w;
  int grid = 0;
  int rc = prepare(op, B, ld, ws, ws_bytes, &w, &grid);
  if (rc != LG_OK) return rc;
  if ((rc = check_ptr(X, op->dtype, "X")) || (rc = check_ptr(G, op->dtype, "G")) ||
      (rc = check_ptr(gX, op->dtype, "gX")))
    return rc;
  if (!g_params) return fail("lg_slq_apply_vjp: null g_params");
  if (gX == X || gX == G) return fail("lg_slq_apply_vjp: gX must not alias X or G");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define LG_VJP(TT, L, NS, NP)                                                                                       \
  apply_vjp_t<TT, L, NS>(*op, B, ld, static_cast<const TT*>(X), static_cast<const TT*>(G), static_cast<TT*>(gX), \
                     g_params, w, grid, st)
  cudaError_t e = LG_DISPATCH(op->dtype, B, LG_VJP);
#undef LG_VJP
  return e == cudaSuccess ? LG_OK : cuda_fail("lg_slq_apply_vjp", e);
}

extern "C" int lg_slq_small_side(int B, int m, int func, int mode, const double* alpha, const double* beta,
                                 const double* znorm, const double* gu, double g_scale, double* out, double* g_alpha,
                                 double* g_beta, int* status, void* ws, size_t ws_bytes, void* stream) {
  if (B < 1 || B > kMaxB) return fail("lg_slq_small_side: B must be in [1, 128]");
  if (m < 1 || m > kMaxCols) return fail("lg_slq_small_side: m must be in [1, 128]");
  if (func < LG_FUNC_LOG || func > LG_FUNC_INV) return fail("lg_slq_small_side: unknown func");
  if (mode < 0 || mode > 2) return fail("lg_slq_small_side: mode must be 0, 1 or 2");
  if (!alpha || !beta || !status || (mode == 0 && !znorm) || (mode == 2 && !gu) || (mode != 2 && !out) ||
      (mode != 1 && (!g_alpha || !g_beta)))
    return fail("lg_slq_small_side: null argument");
  const int grid = slq_grid();
  int rc = check_ws(ws, ws_bytes, ws_layout(0, 0, 4, B, 1, grid, nullptr, nullptr));
  if (rc != LG_OK) return rc;
  Ws w;
  ws_layout(0, 0, 4, B, 1, grid, static_cast<char*>(ws), &w);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t smem = (size_t)m * m * sizeof(double);
  cudaError_t e = cudaFuncSetAttribute(small_side_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) {
    small_side_kernel<<<B, kQT, smem, st>>>(m, func, mode, alpha, beta, znorm, gu, g_scale, out, g_alpha, g_beta,
                                            w.qscr, status);
    e = cudaGetLastError();
  }
  return e == cudaSuccess ? LG_OK : cuda_fail("lg_slq_small_side", e);
}

// ---- block steps around a caller-formed product ------------------------------
static int prepare_block(int n, int B, int ld, int dtype, void* ws, size_t ws_bytes, Ws* w, int* grid) {
  int rc = check_block(n, B, ld, dtype);
  if (rc != LG_OK) return rc;
  *grid = slq_grid();
  rc = check_ws(ws, ws_bytes, ws_layout(0, 0, 4, B, 1, *grid, nullptr, nullptr));
  if (rc != LG_OK) return rc;
  ws_layout(0, 0, 4, B, 1, *grid, static_cast<char*>(ws), w);
  return LG_OK;
}

extern "C" int lg_slq_block_start(int n, int B, int ld, int dtype, const void* Z, void* V0, double* znorm, void* ws,
                                  size_t ws_bytes, void* stream) {
  Ws w;
  int grid = 0;
  int rc = prepare_block(n, B, ld, dtype, ws, ws_bytes, &w, &grid);
  if (rc != LG_OK) return rc;
  if ((rc = check_ptr(Z, dtype, "Z")) || (rc = check_ptr(V0, dtype, "V0"))) return rc;
  if (!znorm) return fail("lg_slq_block_start: null znorm");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = reset_counters(w, st);
  if (e == cudaSuccess) {
#define LG_START(TT, L, NS, NP)                                                                                     \
  (coldot_kernel<TT, L, NS><<<grid, kT, 0, st>>>(n, ld, B, static_cast<const TT*>(Z), nullptr, w.cs[0]),         \
   normalize_kernel<TT, L, NS><<<grid, kT, 0, st>>>(n, ld, B, static_cast<const TT*>(Z), w.cs[0].out,            \
                                                static_cast<TT*>(V0), znorm, 1),                            \
   cudaGetLastError())
    e = LG_DISPATCH(dtype, B, LG_START);
#undef LG_START
  }
  return e == cudaSuccess ? LG_OK : cuda_fail("lg_slq_block_start", e);
}

extern "C" int lg_slq_block_step(int n, int B, int ld, int dtype, int j, int m, const void* W, const void* Vj,
                                 const void* Vjm1, void* R, void* Vnext, double* alpha, double* beta, void* ws,
                                 size_t ws_bytes, void* stream) {
  Ws w;
  int grid = 0;
  int rc = prepare_block(n, B, ld, dtype, ws, ws_bytes, &w, &grid);
  if (rc != LG_OK) return rc;
  if (j < 0 || j >= m || m > kMaxCols) return fail("lg_slq_block_step: need 0 <= j < m <= 128");
  if ((rc = check_ptr(W, dtype, "W")) || (rc = check_ptr(Vj, dtype, "Vj")) || (rc = check_ptr(R, dtype, "R")) ||
      (rc = check_ptr(Vnext, dtype, "Vnext")))
    return rc;
  if (j > 0 && (rc = check_ptr(Vjm1, dtype, "Vjm1"))) return rc;
  if (!alpha || !beta) return fail("lg_slq_block_step: null alpha/beta");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define LG_STEP(TT, L, NS, NP)                                                                                          \
  (coldot_kernel<TT, L, NS><<<grid, kT, 0, st>>>(n, ld, B, static_cast<const TT*>(Vj), static_cast<const TT*>(W),    \
                                             w.cs[0]),                                                          \
   recur_kernel<TT, L, NS><<<grid, kT, 0, st>>>(n, ld, B, j, m, static_cast<const TT*>(W), static_cast<const TT*>(Vj), \
                                            j > 0 ? static_cast<const TT*>(Vjm1) : nullptr, w.cs[0].out, alpha, \
                                            beta, static_cast<TT*>(R), w.cs[1]),                                \
   normalize_kernel<TT, L, NS><<<grid, kT, 0, st>>>(n, ld, B, static_cast<const TT*>(R), w.cs[1].out,               \
                                                static_cast<TT*>(Vnext), beta + j, m),                          \
   cudaGetLastError())
  cudaError_t e = LG_DISPATCH(dtype, B, LG_STEP);
#undef LG_STEP
  return e == cudaSuccess ? LG_OK : cuda_fail("lg_slq_block_step", e);
}

extern "C" int lg_slq_block_lambda(int n, int B, int ld, int dtype, int j, int m, const void* xi, const void* xplus,
                                   const void* xj, const double* beta, const double* g_alpha, const double* g_beta,
                                   const double* g_out, void* lam, void* ws, size_t ws_bytes, void* stream) {
  Ws w;
  int grid = 0;
  int rc = prepare_block(n, B, ld, dtype, ws, ws_bytes, &w, &grid);
  if (rc != LG_OK) return rc;
  if (j < 0 || j >= m || m > kMaxCols) return fail("lg_slq_block_lambda: need 0 <= j < m <= 128");
  if ((rc = check_ptr(xplus, dtype, "xplus")) || (rc = check_ptr(xj, dtype, "xj")) ||
      (rc = check_ptr(lam, dtype, "lam")))
    return rc;
  if (xi && (rc = check_ptr(xi, dtype, "xi"))) return rc;
  if (!beta || !g_alpha || !g_beta) return fail("lg_slq_block_lambda: null scalar arrays");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // xi == NULL starts the sweep (xi = 0, no dots from a previous step)
#define LG_LAM(TT, L, NS, NP)                                                                                              \
  (lam_kernel<TT, L, NS><<<grid, kT, 0, st>>>(n, ld, B, j, m, static_cast<const TT*>(xi), static_cast<const TT*>(xplus), \
                                          static_cast<const TT*>(xj), xi ? w.cs[1].out : nullptr, g_alpha, g_beta,  \
                                          g_out, beta, static_cast<TT*>(lam), w.munu),                             \
   cudaGetLastError())
  cudaError_t e = LG_DISPATCH(dtype, B, LG_LAM);
#undef LG_LAM
  return e == cudaSuccess ? LG_OK : cuda_fail("lg_slq_block_lambda", e);
}

extern "C" int lg_slq_block_xi(int n, int B, int ld, int dtype, int j, int m, const void* Plam, const void* lam,
                               const void* lplus, const void* xplus, const void* xj, const void* xjm1,
                               const double* alpha, const double* beta, const double* dcoef, const void* G, void* xi,
                               void* ws, size_t ws_bytes, void* stream) {
  Ws w;
  int grid = 0;
  int rc = prepare_block(n, B, ld, dtype, ws, ws_bytes, &w, &grid);
  if (rc != LG_OK) return rc;
  if (j < 0 || j >= m || m > kMaxCols) return fail("lg_slq_block_xi: need 0 <= j < m <= 128");
  if ((rc = check_ptr(Plam, dtype, "Plam")) || (rc = check_ptr(lam, dtype, "lam")) ||
      (rc = check_ptr(xplus, dtype, "xplus")) || (rc = check_ptr(xj, dtype, "xj")) ||
      (rc = check_ptr(xi, dtype, "xi")))
    return rc;
  if (lplus && (rc = check_ptr(lplus, dtype, "lplus"))) return rc;
  if (xjm1 && (rc = check_ptr(xjm1, dtype, "xjm1"))) return rc;
  if ((dcoef == nullptr) != (G == nullptr)) return fail("lg_slq_block_xi: dcoef and G go together");
  if (G && (rc = check_ptr(G, dtype, "G"))) return rc;
  if (!alpha || !beta) return fail("lg_slq_block_xi: null alpha/beta");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = (xjm1 ? reset_counters(w, st) : cudaSuccess);
  if (e == cudaSuccess) {
#define LG_XI(TT, L, NS, NP)                                                                                               \
  (xi_kernel<TT, L, NS><<<grid2(), kT, 0, st>>>(n, ld, B, j, m, static_cast<const TT*>(Plam), static_cast<const TT*>(lam), \
                                         static_cast<const TT*>(lplus), static_cast<const TT*>(xplus),             \
                                         static_cast<const TT*>(xj), static_cast<const TT*>(xjm1), alpha, beta,    \
                                         w.munu, dcoef, static_cast<const TT*>(G), static_cast<TT*>(xi), w.cs[1]), \
   cudaGetLastError())
    e = LG_DISPATCH(dtype, B, LG_XI);
#undef LG_XI
  }
  return e == cudaSuccess ? LG_OK : cuda_fail("lg_slq_block_xi", e);
}

extern "C" int lg_slq_block_start_grad(int n, int B, int ld, int dtype, const void* xi, const void* V0, const void* Z,
                                       const double* znorm, const double* g_znorm, void* gZ, void* ws,
                                       size_t ws_bytes, void* stream) {
  Ws w;
  int grid = 0;
  int rc = prepare_block(n, B, ld, dtype, ws, ws_bytes, &w, &grid);
  if (rc != LG_OK) return rc;
  if ((rc = check_ptr(xi, dtype, "xi")) || (rc = check_ptr(V0, dtype, "V0")) || (rc = check_ptr(Z, dtype, "Z")) ||
      (rc = check_ptr(gZ, dtype, "gZ")))
    return rc;
  if (!znorm) return fail("lg_slq_block_start_grad: null znorm");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = reset_counters(w, st);
  if (e == cudaSuccess) {
#define LG_SG(TT, L, NS, NP)                                                                                              \
  (coldot_kernel<TT, L, NS><<<grid, kT, 0, st>>>(n, ld, B, static_cast<const TT*>(xi), static_cast<const TT*>(V0),     \
                                             w.cs[0]),                                                            \
   start_grad_kernel<TT, L, NS><<<grid, kT, 0, st>>>(n, ld, B, static_cast<const TT*>(xi), static_cast<const TT*>(V0), \
                                                 static_cast<const TT*>(Z), znorm, g_znorm, w.cs[0].out,          \
                                                 static_cast<TT*>(gZ)),                                           \
   cudaGetLastError())
    e = LG_DISPATCH(dtype, B, LG_SG);
#undef LG_SG
  }
  return e == cudaSuccess ? LG_OK : cuda_fail("lg_slq_block_start_grad", e);
}

extern "C" int lg_dense_matvec(int n, int dtype, const void* A, const void* x, int ldx, void* y, int ldy,
                               void* stream) {
  if (n < 1 || ldx < 1 || ldy < 1 || !A || !x || !y) return fail("lg_dense_matvec: invalid arguments");
  if (dtype != LG_F32 && dtype != LG_F64) return fail("lg_dense_matvec: dtype must be LG_F32 or LG_F64");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = slq_grid();
  if (dtype == LG_F64)
    dense_matvec_kernel<double><<<grid, kT, 0, st>>>(n, static_cast<const double*>(A), static_cast<const double*>(x),
                                                     ldx, static_cast<double*>(y), ldy);
  else
    dense_matvec_kernel<float><<<grid, kT, 0, st>>>(n, static_cast<const float*>(A), static_cast<const float*>(x), ldx,
                                                    static_cast<float*>(y), ldy);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LG_OK : cuda_fail("lg_dense_matvec", e);
}

extern "C" int lg_outer_accumulate(int n, int dtype, const void* lam, const void* x, int ld, double* gA,
                                   void* stream) {
  if (n < 1 || ld < 1 || !lam || !x || !gA) return fail("lg_outer_accumulate: invalid arguments");
  if (dtype != LG_F32 && dtype != LG_F64) return fail("lg_outer_accumulate: dtype must be LG_F32 or LG_F64");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = slq_grid() * 2;
  if (dtype == LG_F64)
    outer_acc_kernel<double><<<grid, 256, 0, st>>>(n, ld, static_cast<const double*>(lam),
                                                    static_cast<const double*>(x), gA);
  else
    outer_acc_kernel<float><<<grid, 256, 0, st>>>(n, ld, static_cast<const float*>(lam), static_cast<const float*>(x),
                                                   gA);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LG_OK : cuda_fail("lg_outer_accumulate", e);
}
