// advopt_adam_step_noalloc: the Adam-family step of one tensor for callers
// that cannot allocate device memory.
//
// The ordinary entry point (advopt_adam_step) expects the caller to hand it
// device buffers for the descriptor table, the CTA plan and the factored
// column partials.  A caller that works inside a fixed memory budget it
// cannot grow — a runtime with its own pre-sized device arena and no
// allocator hook, or code that must not call cudaMalloc (or a framework's
// caching allocator) in the middle of a training step — has nowhere to put
// that scratch.  This variant keeps it in a file-scope __device__ array of
// ADVOPT_NOALLOC_SCRATCH_BYTES that every GPU which loads the library holds
// until the process exits; the caller passes only its own tensors.
//
// Set-up: the first call on a device looks up the array's device address with
// cudaGetSymbolAddress (with that device current) and caches it; make that
// first call before any stream capture.  All calls share the one array and it
// keeps the last call's contents: every call rewrites the descriptor, the plan
// and the error word before its kernels read them, and the kernels overwrite
// every column partial they later sum, so nothing needs to start at zero.  A
// CTA whose bounded wait gives up leaves its partials unwritten; the error
// word then stops the factored finish, which leaves the factors unchanged.
// Without launch->err that word is the array's own, which no caller reads:
// callers that need to know pass their own device word in launch->err.
// Calls whose kernels overlap on the GPU (other streams, or other host threads
// on the same device) race on the array and must be serialised by the caller.
//
// Kernel choice, shared memory and the fast kernel's limits follow the host
// planner of the optimizer classes (32-bit element offsets below 2^34
// elements; factored tensors wider than 8192 columns accumulate their column
// partials in the array instead of shared memory).  One difference: the plan
// is one piece per CTA, so a factored tensor's float32 column partials sum
// up to d1 / grid rows before the float64 reduction (the planner cuts pieces
// at 64 rows); on the Llama embedding's 24576 x 21376 effective shape, where
// the array caps the grid near 195 CTAs, that is 126 rows.
#include <cstdio>
#include <mutex>

#include "advopt.h"
#include "capi_internal.h"
#include "common.cuh"

namespace advopt {
namespace {

__device__ __align__(256) unsigned char g_noalloc_scratch[ADVOPT_NOALLOC_SCRATCH_BYTES];

std::mutex g_mu;
constexpr int kMaxDevices = 128;
void* g_base[kMaxDevices] = {};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Columns of the fast kernel's shared-memory column accumulator (the host
// planner's FAST_COLS).
constexpr int kNoallocFastCols = 8192;

inline int64_t gcd64(int64_t a, int64_t b) {
  while (b) {
    const int64_t r = a % b;
    a = b;
    b = r;
  }
  return a;
}

struct ScratchLayout {
  size_t desc = 0, index = 0, pieces = 0, offsets = 0, err = 0, partial = 0, total = 0;
};

ScratchLayout layout_for(int grid, int64_t d2_partial) {
  ScratchLayout l;
  size_t off = 0;
  l.desc = off;
  off = align256(off + sizeof(advopt_adam_tensor));
  l.index = off;
  off = align256(off + sizeof(int32_t));
  l.pieces = off;
  off = align256(off + (size_t)grid * sizeof(advopt_piece));
  l.offsets = off;
  off = align256(off + (size_t)(grid + 1) * sizeof(int32_t));
  l.err = off;
  off = align256(off + sizeof(int32_t));
  l.partial = off;
  off = align256(off + (size_t)grid * (size_t)d2_partial * sizeof(float));
  l.total = off;
  return l;
}

// Writes the descriptor, a one-piece-per-CTA plan (cut points c*n/grid snapped
// to the nearest multiple of `unit`) and clears the error word.
__global__ void noalloc_prepare_kernel(advopt_adam_tensor t, unsigned char* base, int grid, int64_t unit,
                                       ScratchLayout l) {
  const int64_t n = t.numel;
  auto cut = [&](int c) -> int64_t {
    if (c <= 0) return 0;
    if (c >= grid) return n;
    const int64_t x = (int64_t)((__int128)c * n / grid);
    const int64_t down = (x / unit) * unit;
    const int64_t up = min(n, down + unit);
    return (x - down <= up - x) ? down : up;
  };
  if (threadIdx.x == 0) {
    t.col_partial = (t.flags & ADVOPT_T_FACTORED) ? reinterpret_cast<float*>(base + l.partial) : nullptr;
    t.slot_base = 0;
    t.n_slots = grid;
    *reinterpret_cast<advopt_adam_tensor*>(base + l.desc) = t;
    *reinterpret_cast<int32_t*>(base + l.index) = 0;
    *reinterpret_cast<int32_t*>(base + l.err) = 0;
  }
  advopt_piece* pieces = reinterpret_cast<advopt_piece*>(base + l.pieces);
  int32_t* offs = reinterpret_cast<int32_t*>(base + l.offsets);
  for (int c = threadIdx.x; c <= grid; c += blockDim.x) {
    offs[c] = c;
    if (c < grid) {
      advopt_piece pc;
      pc.begin = cut(c);
      pc.end = cut(c + 1);
      pc.tensor = 0;
      pc.slot = c;
      pieces[c] = pc;
    }
  }
}

int scratch_base(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return check_cuda(e, "advopt_adam_step_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return set_error(ADVOPT_E_INVALID, "advopt_adam_step_noalloc: device ordinal");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_base[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return check_cuda(e, "advopt_adam_step_noalloc: cudaGetSymbolAddress");
    g_base[dev] = p;
  }
  *out = g_base[dev];
  return ADVOPT_OK;
}

}  // namespace
}  // namespace advopt

using namespace advopt;

extern "C" int advopt_adam_step_noalloc(const advopt_adam_tensor* tensor, const advopt_adam_launch* launch,
                                        void* stream) {
  if (!tensor || !launch) return set_error(ADVOPT_E_INVALID, "advopt_adam_step_noalloc: null argument");
  const advopt_adam_tensor& t = *tensor;
  const advopt_adam_launch& hp = *launch;
  if (t.numel <= 0) return ADVOPT_OK;
  if (hp.precision < 0 || hp.precision > 3 || hp.algo < 0 || hp.algo > 1 || hp.param_dtype < 0 ||
      hp.param_dtype > 1)
    return set_error(ADVOPT_E_INVALID,
                     "advopt_adam_step_noalloc: precision/dtype code out of range, or an algorithm other than "
                     "AdamW / auxiliary Adam (Prodigy needs per-launch statistics buffers)");
  if (hp.flags & (ADVOPT_F_FISHER | ADVOPT_F_FISHER_STATS | ADVOPT_F_PRODIGY_STATS))
    return set_error(ADVOPT_E_INVALID, "advopt_adam_step_noalloc: Fisher weight decay is not supported here");
  // per-piece grad sums would index pieces the caller never sees; a dynamic
  // beta2 (layer_beta2 / layer_of_tensor[0]) passes through unchanged
  if (hp.flags & ADVOPT_F_GRAD_SQ)
    return set_error(ADVOPT_E_INVALID, "advopt_adam_step_noalloc: per-piece grad sums are not supported here");
  if (hp.layer_beta2 && !hp.layer_of_tensor)
    return set_error(ADVOPT_E_INVALID, "advopt_adam_step_noalloc: layer_beta2 without layer_of_tensor");
  if ((hp.flags & (ADVOPT_F_FACT_M | ADVOPT_F_EMIT_UPDATE)) || (t.flags & ADVOPT_T_FACT_M))
    return set_error(ADVOPT_E_INVALID,
                     "advopt_adam_step_noalloc: factored momentum and update emission are not supported here");
  const bool fact = t.flags & ADVOPT_T_FACTORED;
  const int64_t d2 = fact ? t.d2 : 0;
  if (fact && (t.d1 <= 0 || d2 <= 0 || t.d1 * d2 != t.numel))
    return set_error(ADVOPT_E_INVALID, "advopt_adam_step_noalloc: factored shape does not match numel");

  void* base_v = nullptr;
  int rc = scratch_base(&base_v);
  if (rc != ADVOPT_OK) return rc;
  unsigned char* base = static_cast<unsigned char*>(base_v);
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  // kernel choice and shared memory, as the Python planner does it
  const bool ext = hp.flags & (ADVOPT_F_ATAN2 | ADVOPT_F_NORMED | ADVOPT_F_ANCHORS);
  const bool ffast = !fact || (d2 >= 2048 && d2 % 8 == 0 && (reinterpret_cast<uintptr_t>(t.col_factor) % 16) == 0 &&
                               (reinterpret_cast<uintptr_t>(t.row_factor) % 16) == 0);
  int gen_offset = fact ? (int)((d2 + 3) / 4 * 4) : 0;
  int stages = 0, smem_floats = 0;
  // the fast kernel keeps element offsets in 32 bits
  const bool fast = !ext && ffast && t.numel < (int64_t(1) << 34);
  if (fast) {
    // factored tensors wider than the shared-memory accumulator keep their
    // column partials in their slot rows of the array
    if (gen_offset > kNoallocFastCols) gen_offset = kNoallocFastCols;
    const int bpp = hp.param_dtype == ADVOPT_DT_BF16 ? 2 : 4;
    int bps = 4;
    if (hp.precision == ADVOPT_PREC_INT8_SR) bps = 1;
    else if (hp.precision == ADVOPT_PREC_BF16_SR || (hp.precision == ADVOPT_PREC_AUTO && bpp == 2)) bps = 2;
    const int stage = 2048 * (2 * bpp + 2 * bps);
    int st = (112 * 1024 - gen_offset * 4) / stage;
    stages = st < 2 ? 2 : (st > 4 ? 4 : st);
    smem_floats = gen_offset + stages * stage / 4;
  } else {
    smem_floats = gen_offset + ((fact && !ffast) ? 2 * 2048 + 4 : 0);
  }
  if (smem_floats > 56832)
    return set_error(ADVOPT_E_INVALID, "advopt_adam_step_noalloc: factored d2 too large for shared memory");
  int dev = 0, sms = 0, ctas = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = run_occupancy(hp.precision, hp.param_dtype, hp.algo, smem_floats, &ctas, fast ? 1 : 0);
  if (e != cudaSuccess) return check_cuda(e, "advopt_adam_step_noalloc: occupancy");
  if (ctas < 1) ctas = 1;
  const int64_t unit = fact ? d2 * 2048 / gcd64(d2, 2048) : 2048;
  const int64_t units = (t.numel + unit - 1) / unit;
  int64_t grid = (int64_t)sms * ctas;
  if (grid > units) grid = units;
  // the column partials (grid rows of d2 floats) must fit in the array
  const int64_t fixed = (int64_t)layout_for(0, 0).total + 64 * 1024;
  if (fact) {
    const int64_t per = d2 * (int64_t)sizeof(float) + (int64_t)sizeof(advopt_piece) + 8;
    const int64_t cap = ((int64_t)ADVOPT_NOALLOC_SCRATCH_BYTES - fixed) / per;
    if (cap < 1) {
      char msg[256];
      std::snprintf(msg, sizeof(msg),
                    "advopt_adam_step_noalloc: factored d2 = %lld needs more than the %u-byte scratch array",
                    (long long)d2, (unsigned)ADVOPT_NOALLOC_SCRATCH_BYTES);
      return set_error(ADVOPT_E_INVALID, msg);
    }
    if (grid > cap) grid = cap;
  }
  if (grid < 1) grid = 1;
  const ScratchLayout l = layout_for((int)grid, fact ? d2 : 0);
  if (l.total > ADVOPT_NOALLOC_SCRATCH_BYTES) {
    char msg[256];
    std::snprintf(msg, sizeof(msg), "advopt_adam_step_noalloc: needs %zu bytes of scratch, the array holds %u",
                  l.total, (unsigned)ADVOPT_NOALLOC_SCRATCH_BYTES);
    return set_error(ADVOPT_E_INVALID, msg);
  }

  noalloc_prepare_kernel<<<1, 256, 0, s>>>(t, base, (int)grid, unit, l);
  e = cudaGetLastError();
  if (e != cudaSuccess) return check_cuda(e, "advopt_adam_step_noalloc: prepare");

  advopt_adam_launch L = hp;
  L.tensors = reinterpret_cast<const advopt_adam_tensor*>(base + l.desc);
  L.pieces = reinterpret_cast<const advopt_piece*>(base + l.pieces);
  L.cta_offsets = reinterpret_cast<const int32_t*>(base + l.offsets);
  L.piece_stats = nullptr;
  L.piece_gsq = nullptr;
  // a caller-supplied error word (launch->err) is honoured; otherwise the
  // array's own word records a bounded wait that gave up
  L.err = hp.err ? hp.err : reinterpret_cast<int32_t*>(base + l.err);
  L.n_tensors = 1;
  L.n_pieces = (int32_t)grid;
  L.grid = (int32_t)grid;
  L.smem_floats = smem_floats;
  L.gen_offset = gen_offset;
  L.stages = stages;
  e = run_adam(L, s);
  if (e != cudaSuccess) return check_cuda(e, "advopt_adam_step_noalloc: step");
  if (fact) {
    e = run_factored_finish(L.tensors, reinterpret_cast<const int32_t*>(base + l.index), 1, (int)d2, L.err, s);
    if (e != cudaSuccess) return check_cuda(e, "advopt_adam_step_noalloc: factored finish");
  }
  return ADVOPT_OK;
}
