// A C++ caller of the six custom-call targets the reference lowers to kernels
// (iree_metal/patches/08-gemm-dispatch-pass.patch:57-123, 230-236), written
// against include/nl_ops.h alone and linked with libnl_ops.so, the way an
// XLA FFI handler or any other native host would bind them.  Operand order and
// dtypes are the reference's:
//   flash_attention_fwd      Q, K, V f32 [n,s,d]             -> O f32, L f32 [n,s]
//   flash_attention_bwd_dq   Q, K, V, dO f32, L, D f32 [n,s] -> dQ f32
//   flash_attention_bwd_dkdv Q, K, V, dO f32, L, D f32       -> dK, dV f32
//   gemm                     A bf16 [M,K], B bf16 [K,N]      -> C f32 [M,N]
//   ce_fwd                   logits f32 [M,V], targets i32   -> loss f32 [M], lse f32 [M]
//   ce_bwd                   logits, targets, lse            -> dlogits f32 [M,V] (/ M)
// Each result is compared with a double-precision host computation.  Prints
// one line per target and exits 0 only if all six pass.  Test infrastructure.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include <cuda_runtime.h>

#include "nl_ops.h"

namespace {

struct Rng {
  uint64_t s;
  explicit Rng(uint64_t seed) : s(seed * 0x9E3779B97F4A7C15ull + 1) {}
  double uniform() {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    return ((s >> 11) + 0.5) * (1.0 / 9007199254740992.0);
  }
  float normal() { return static_cast<float>(std::sqrt(-2.0 * std::log(uniform())) * std::cos(6.283185307179586 * uniform())); }
};

uint16_t to_bf16(float f) {  // round to nearest even
  uint32_t u;
  std::memcpy(&u, &f, 4);
  u += 0x7fff + ((u >> 16) & 1);
  return static_cast<uint16_t>(u >> 16);
}
float from_bf16(uint16_t h) {
  uint32_t u = static_cast<uint32_t>(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

template <typename T>
T* dev_copy(const std::vector<T>& h) {
  T* d = nullptr;
  if (cudaMalloc(&d, h.size() * sizeof(T)) != cudaSuccess) return nullptr;
  cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice);
  return d;
}
template <typename T>
std::vector<T> host_copy(const T* d, size_t n) {
  std::vector<T> h(n);
  cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost);
  return h;
}

double nrel(const std::vector<float>& a, const std::vector<double>& b) {
  double e = 0, m = 1e-12;
  for (size_t i = 0; i < a.size(); ++i) {
    e = std::fmax(e, std::fabs(a[i] - b[i]));
    m = std::fmax(m, std::fabs(b[i]));
  }
  return e / m;
}

int failures = 0;
void report(const char* target, double err, double tol, int status) {
  const bool ok = status == NL_OK && err <= tol;
  std::printf("%-26s status %d  max|err|/max|ref| %.3e  (tol %.0e)  %s\n", target, status, err, tol,
              ok ? "PASS" : "FAIL");
  if (!ok) ++failures;
}

}  // namespace

int main() {
  const int n = 3, s = 200, d = 64;
  const size_t E = static_cast<size_t>(n) * s * d;
  Rng rng(7);
  std::vector<float> Q(E), K(E), V(E), dO(E);
  for (auto* v : {&Q, &K, &V, &dO})
    for (auto& x : *v) x = rng.normal();

  // ---- host reference (double): P = softmax(scale * Q K^T, causal), O = P V,
  // dP = dO V^T, D = rowsum(dO * O), dS = P (dP - D), dQ = scale dS K,
  // dK = scale dS^T Q, dV = P^T dO.
  const double scale = 1.0 / std::sqrt(static_cast<double>(d));
  std::vector<double> Or(E, 0), Lr(n * s), dQr(E, 0), dKr(E, 0), dVr(E, 0);
  for (int h = 0; h < n; ++h) {
    const size_t b = static_cast<size_t>(h) * s * d;
    std::vector<double> P(static_cast<size_t>(s) * s, 0.0);
    for (int i = 0; i < s; ++i) {
      double mx = -1e300;
      for (int j = 0; j <= i; ++j) {
        double a = 0;
        for (int k = 0; k < d; ++k) a += static_cast<double>(Q[b + i * d + k]) * K[b + j * d + k];
        P[i * s + j] = a * scale;
        mx = std::fmax(mx, P[i * s + j]);
      }
      double sum = 0;
      for (int j = 0; j <= i; ++j) sum += std::exp(P[i * s + j] - mx);
      Lr[h * s + i] = mx + std::log(sum);
      for (int j = 0; j <= i; ++j) P[i * s + j] = std::exp(P[i * s + j] - Lr[h * s + i]);
      for (int j = 0; j <= i; ++j)
        for (int k = 0; k < d; ++k) Or[b + i * d + k] += P[i * s + j] * V[b + j * d + k];
    }
    for (int i = 0; i < s; ++i) {
      double Dd = 0;
      for (int k = 0; k < d; ++k) Dd += dO[b + i * d + k] * Or[b + i * d + k];
      for (int j = 0; j <= i; ++j) {
        double dp = 0;
        for (int k = 0; k < d; ++k) dp += static_cast<double>(dO[b + i * d + k]) * V[b + j * d + k];
        const double ds = P[i * s + j] * (dp - Dd);
        for (int k = 0; k < d; ++k) {
          dQr[b + i * d + k] += scale * ds * K[b + j * d + k];
          dKr[b + j * d + k] += scale * ds * Q[b + i * d + k];
          dVr[b + j * d + k] += P[i * s + j] * dO[b + i * d + k];
        }
      }
    }
  }

  float *dQin = dev_copy(Q), *dKin = dev_copy(K), *dVin = dev_copy(V), *ddO = dev_copy(dO);
  float *dOut, *dL, *dD, *ddQ, *ddK, *ddV;
  cudaMalloc(&dOut, E * 4);
  cudaMalloc(&dL, n * s * 4);
  cudaMalloc(&dD, n * s * 4);
  cudaMalloc(&ddQ, E * 4);
  cudaMalloc(&ddK, E * 4);
  cudaMalloc(&ddV, E * 4);
  size_t wsb = 0;
  for (int t = 0; t < 3; ++t) wsb = std::max(wsb, nl_flash_attention_workspace_bytes(t, n, s, d, NL_F32));
  void* ws = nullptr;
  cudaMalloc(&ws, wsb);
  cudaStream_t st = nullptr;

  // flash_attention_fwd
  int rc = nl_flash_attention_fwd_dt(dQin, dKin, dVin, dOut, dL, n, s, d, NL_F32, ws, wsb, st);
  cudaDeviceSynchronize();
  auto O = host_copy(dOut, E);
  auto L = host_copy(dL, n * s);
  double lerr = 0;
  for (int i = 0; i < n * s; ++i) lerr = std::fmax(lerr, std::fabs(L[i] - Lr[i]));
  report("flash_attention_fwd", std::fmax(nrel(O, Or), lerr / 2.0), 1e-2, rc);

  // D = rowsum(dO * O) by the caller, as nlearn/attention.py:115 does
  std::vector<float> D(n * s);
  for (int r = 0; r < n * s; ++r) {
    double a = 0;
    for (int k = 0; k < d; ++k) a += static_cast<double>(dO[r * d + k]) * O[r * d + k];
    D[r] = static_cast<float>(a);
  }
  cudaMemcpy(dD, D.data(), n * s * 4, cudaMemcpyHostToDevice);
  rc = nl_flash_attention_bwd_dq_dt(dQin, dKin, dVin, ddO, dL, dD, ddQ, n, s, d, NL_F32, ws, wsb, st);
  cudaDeviceSynchronize();
  report("flash_attention_bwd_dq", nrel(host_copy(ddQ, E), dQr), 1e-2, rc);
  rc = nl_flash_attention_bwd_dkdv_dt(dQin, dKin, dVin, ddO, dL, dD, ddK, ddV, n, s, d, NL_F32, ws, wsb, st);
  cudaDeviceSynchronize();
  const double ek = nrel(host_copy(ddK, E), dKr), ev = nrel(host_copy(ddV, E), dVr);
  report("flash_attention_bwd_dkdv", std::fmax(ek, ev), 1e-2, rc);

  // gemm: A bf16 [M,K] . B bf16 [K,N] -> C f32 (padded sizes of the reference ABI)
  const int M = 96, N = 96, Kd = 128;
  std::vector<uint16_t> A(M * Kd), B(Kd * N);
  std::vector<float> Af(M * Kd), Bf(Kd * N);
  for (int i = 0; i < M * Kd; ++i) Af[i] = from_bf16(A[i] = to_bf16(rng.normal()));
  for (int i = 0; i < Kd * N; ++i) Bf[i] = from_bf16(B[i] = to_bf16(rng.normal()));
  std::vector<double> Cr(M * N, 0);
  for (int i = 0; i < M; ++i)
    for (int k = 0; k < Kd; ++k)
      for (int j = 0; j < N; ++j) Cr[i * N + j] += static_cast<double>(Af[i * Kd + k]) * Bf[k * N + j];
  uint16_t *dA = dev_copy(A), *dB = dev_copy(B);
  float* dC;
  cudaMalloc(&dC, M * N * 4);
  rc = nl_gemm(dA, dB, dC, M, N, Kd, st);
  cudaDeviceSynchronize();
  report("gemm", nrel(host_copy(dC, M * N), Cr), 1e-5, rc);

  // ce_fwd / ce_bwd on f32 logits
  const int Mc = 64, Vc = 1000;
  std::vector<float> lg(Mc * Vc);
  std::vector<int> tg(Mc);
  for (auto& x : lg) x = 2.f * rng.normal();
  for (auto& t : tg) t = static_cast<int>(rng.uniform() * Vc) % Vc;
  std::vector<double> lossr(Mc), lser(Mc), dlr(Mc * Vc);
  for (int r = 0; r < Mc; ++r) {
    double mx = -1e300, sum = 0;
    for (int v = 0; v < Vc; ++v) mx = std::fmax(mx, lg[r * Vc + v]);
    for (int v = 0; v < Vc; ++v) sum += std::exp(lg[r * Vc + v] - mx);
    lser[r] = mx + std::log(sum);
    lossr[r] = lser[r] - lg[r * Vc + tg[r]];
    for (int v = 0; v < Vc; ++v) dlr[r * Vc + v] = (std::exp(lg[r * Vc + v] - lser[r]) - (v == tg[r])) / Mc;
  }
  float* dlg = dev_copy(lg);
  int* dtg = dev_copy(tg);
  float *dloss, *dlse, *ddl;
  cudaMalloc(&dloss, Mc * 4);
  cudaMalloc(&dlse, Mc * 4);
  cudaMalloc(&ddl, Mc * Vc * 4);
  rc = nl_ce_fwd(dlg, Vc, NL_F32, dtg, dloss, dlse, Mc, Vc, st);
  cudaDeviceSynchronize();
  const double el = nrel(host_copy(dloss, Mc), lossr), es = nrel(host_copy(dlse, Mc), lser);
  report("ce_fwd", std::fmax(el, es), 1e-5, rc);
  rc = nl_ce_bwd(dlg, Vc, NL_F32, dtg, dlse, ddl, Vc, NL_F32, Mc, Vc, 1.f / Mc, st);
  cudaDeviceSynchronize();
  report("ce_bwd", nrel(host_copy(ddl, Mc * Vc), dlr), 1e-5, rc);

  const int derr = nl_get_device_error(st);
  if (derr != 0) {
    std::printf("device error word %d\n", derr);
    ++failures;
  }
  std::printf("%s: %d of 6 targets failed\n", failures ? "FAIL" : "PASS", failures);
  return failures ? 1 : 0;
}
