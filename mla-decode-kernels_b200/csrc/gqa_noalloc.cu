// Decode entry point for callers that cannot allocate device memory.
//
// gqa_decode_launch needs a caller-provided workspace for the balanced
// schedule's records of the rows it cuts between CTAs and their partial
// softmax states.  Some callers have
// no way to provide one: a host engine that hands all of HBM to its own
// KV-cache pool at start-up and treats any later device allocation as a bug
// (cudaMalloc would synchronise the device mid-step and can fail once the
// pool holds the memory), or a thin foreign-function binding (C, cgo, JNI)
// that has no device allocator to draw a workspace from.  For them,
// gqa_decode_launch_noalloc keeps that scratch in the file-scope array
// below, which the CUDA module reserves on every GPU that loads this library
// and keeps until the process exits.  The entry point itself calls no
// cudaMalloc, cudaFree or other allocating routine.
#include <algorithm>
#include <cstdint>
#include <mutex>

#include "gqa_decode.h"
#include "gqa_internal.h"
#include "gqa_ptx.cuh"

namespace {

constexpr size_t kScratchBytes = GQA_DECODE_NOALLOC_SCRATCH_BYTES;

// Scratch shared by every gqa_decode_launch_noalloc call on a device: the
// balanced schedule's row and CTA records and split partial states, laid out
// per call for its shape.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

struct DeviceState {
  unsigned char* scratch = nullptr;  // device address of g_noalloc_scratch; null until set up
  int sms = 0;
  int smem_attr = 0;
  int occ_threads = 0, occ_smem = 0, occ = 0;
};
constexpr int kMaxDevices = 64;
DeviceState g_state[kMaxDevices];
std::mutex g_mu;

// Set-up for the current device (caller holds g_mu): the scratch array's
// device address (in host code its name is only a stand-in, so it must be
// looked up with this device current) and the SM count.  Only a successful
// set-up is kept; after a failure (e.g. the first call came during a stream
// capture that refused the lookup) the next call tries again.
cudaError_t setup_device(DeviceState* st, int dev) {
  void* ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (e != cudaSuccess) return e;
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  st->sms = sms;
  st->scratch = static_cast<unsigned char*>(ptr);
  return cudaSuccess;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" cudaError_t gqa_decode_launch_noalloc(const gqa_bf16* q, const gqa_bf16* k_cache,
                                                 const gqa_bf16* v_cache, const int* block_table,
                                                 const int* seq_lens, gqa_bf16* out, int B,
                                                 int Hq, int Hkv, int block_size, int max_blocks,
                                                 int num_blocks, float scale,
                                                 cudaStream_t stream) {
  gqa::ShapePlan sp;
  if (B < 0 || block_size <= 0 || max_blocks <= 0 || num_blocks < 0 ||
      gqa::make_shape_plan(Hq, Hkv, &sp) != 0)
    return cudaErrorInvalidValue;
  if (B == 0) return cudaSuccess;
  if (!q || !k_cache || !v_cache || !block_table || !seq_lens || !out)
    return cudaErrorInvalidValue;
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out))
    return cudaErrorMisalignedAddress;

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  DeviceState* st = &g_state[dev];
  int grid = 0, sms = 0;
  unsigned char* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (st->scratch == nullptr) {
      e = setup_device(st, dev);
      if (e != cudaSuccess) return e;
    }
    scratch = st->scratch;
    if (st->smem_attr < sp.smem_bytes) {
      e = gqa::scan_kernel_set_smem(sp.smem_bytes);
      if (e != cudaSuccess) return e;
      st->smem_attr = sp.smem_bytes;
    }
    if (st->occ_threads != sp.threads || st->occ_smem != sp.smem_bytes) {
      int o = 0;
      e = gqa::scan_kernel_occupancy(sp.threads, sp.smem_bytes, &o);
      if (e != cudaSuccess) return e;
      if (o < 1) return cudaErrorInvalidConfiguration;
      st->occ_threads = sp.threads;
      st->occ_smem = sp.smem_bytes;
      st->occ = o;
    }
    grid = gqa::balanced_grid(st->sms, st->occ);
    sms = st->sms;
  }

  // Balanced-schedule workspace layout inside the static scratch.  Every
  // region is written before it is read in each call, so nothing needs
  // clearing between calls.
  const gqa::BalancedLayout lay = gqa::balanced_layout(B, sp, grid);
  if (lay.total > kScratchBytes) return cudaErrorInvalidValue;  // shape too large for the scratch

  gqa::ScanParams p{};
  p.q = q;
  p.k = k_cache;
  p.v = v_cache;
  p.block_table = block_table;
  p.seq_lens = seq_lens;
  p.kv_indptr = seq_lens;  // dense page table; the CSR pointers are never read
  p.kv_indices = block_table;
  p.kv_last = seq_lens;
  p.out = out;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.bs = block_size;
  p.max_blocks = max_blocks;
  p.num_blocks = num_blocks;
  p.G = sp.G;
  p.NT = sp.NT;
  p.HG = sp.HG;
  p.NHG = sp.NHG;
  p.ncw = sp.ncw;
  p.row_bytes = sp.row_bytes;
  p.row_stride = sp.row_stride;
  p.stage_bytes = sp.stage_bytes;
  p.nstages = sp.nstages;
  p.out_mode = gqa::kOutBf16;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.wait_ns = gqa::kWaitLimitNs;
  return gqa::launch_balanced_noexchange(p, lay, scratch, sp, sms, grid, stream);
}
