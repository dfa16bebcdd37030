// The controller's per-request shares on the device: the fold of a new audit into the shares it keeps
// per request key (Controller._absorb_audit, observe/controller.py:332-345).
//
// The reference keeps, per request, a float64 share vector. A new audit's row of shares `fresh` with no
// value other than NaN carries no evidence and changes nothing; otherwise new = nan_to_num(fresh) (NaN as
// 0, +-inf as +-DBL_MAX) becomes the request's shares, blended with the ones it had as
// decay * old + (1 - decay) * new. Here the shares live in a ledger, one float64 row per request slot
// (the host maps request keys to slots), and one CTA folds one fresh row: a barrier-OR finds the
// evidence, then every position is blended with each product and the sum rounded on its own, as NumPy
// evaluates the expression (no fused multiply-add).
#include <cfloat>

#include "ekv_common.cuh"

namespace ekv {

constexpr int kLedgerThreads = 256;

struct LedgerParams {
  const void* fresh;  // float or double [rows][fresh_s0]
  int64_t fresh_s0;
  const int32_t* slot;   // [rows] ledger row of the request, < 0: no request
  const uint8_t* blend;  // [rows] != 0: the request has shares to blend with
  double decay;
  int rows, width;
  double* ledger;  // [ledger_rows][ledger_s0]
  int64_t ledger_s0;
  int ledger_rows;
  uint8_t* evidence;  // [rows] out: the row held a value other than NaN (and had a slot)
};

__device__ __forceinline__ double nan_to_num(double x) {
  if (x != x) return 0.0;
  if (x > DBL_MAX) return DBL_MAX;
  if (x < -DBL_MAX) return -DBL_MAX;
  return x;
}

template <typename F>
__global__ void __launch_bounds__(kLedgerThreads) ledger_absorb_kernel(const LedgerParams p) {
  const int r = blockIdx.x, tid = threadIdx.x;
  const int s = p.slot[r];
  if (s < 0 || s >= p.ledger_rows) {
    if (tid == 0) p.evidence[r] = 0;
    return;
  }
  const F* f = static_cast<const F*>(p.fresh) + (int64_t)r * p.fresh_s0;
  int any = 0;
  for (int b = tid; b < p.width && !any; b += kLedgerThreads) any = f[b] == f[b];
  any = __syncthreads_or(any);
  if (tid == 0) p.evidence[r] = any ? 1 : 0;
  if (!any) return;
  double* row = p.ledger + (int64_t)s * p.ledger_s0;
  const double keep = p.decay, take = __dsub_rn(1.0, p.decay);
  if (p.blend[r]) {
    for (int b = tid; b < p.width; b += kLedgerThreads)
      row[b] = __dadd_rn(__dmul_rn(keep, row[b]), __dmul_rn(take, nan_to_num((double)f[b])));
  } else {
    for (int b = tid; b < p.width; b += kLedgerThreads) row[b] = nan_to_num((double)f[b]);
  }
}

}  // namespace ekv

using namespace ekv;

extern "C" int ekv_ledger_absorb(const void* fresh, int fresh_f64, int64_t fresh_stride, const int32_t* slot,
                                 const uint8_t* blend, double decay, int rows, int width, double* ledger,
                                 int64_t ledger_stride, int ledger_rows, uint8_t* evidence, void* stream) {
  clear_error();
  if (!fresh || !slot || !blend || !ledger || !evidence) return fail(EKV_EINVAL, "a required pointer is NULL");
  if (rows <= 0 || width <= 0 || ledger_rows <= 0) return fail(EKV_EINVAL, "rows, width and ledger_rows must be positive");
  if (fresh_stride < width || ledger_stride < width) return fail(EKV_EINVAL, "a row stride is below the width");
  if (!(decay >= 0.0 && decay < 1.0)) return fail(EKV_EINVAL, "the share decay must be in [0, 1)");
  LedgerParams p{fresh, fresh_stride, slot, blend, decay, rows, width, ledger, ledger_stride, ledger_rows, evidence};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (fresh_f64)
    ledger_absorb_kernel<double><<<rows, kLedgerThreads, 0, s>>>(p);
  else
    ledger_absorb_kernel<float><<<rows, kLedgerThreads, 0, s>>>(p);
  return check_launch("ledger_absorb_kernel");
}
