// Allocation-free entry point: fused q/k RMS norm + RoPE + attention on one GPU.
//
// DECLARATION: this entry point is an addition of this project; it has no
// counterpart in the reference project.
//
// Who needs it.  Some callers may not allocate device memory at all: a host
// application that hands every byte of the GPU to its own pool and forbids
// cudaMalloc after start-up, a plugin running inside another framework that
// accounts for all device memory itself, or a latency-critical serving loop
// that must not enter the driver's allocator between requests.  Those callers
// cannot use the heap-backed fused path (ops / parallel.fused), whose kernels
// stage q/k/v in a receive buffer obtained from cudaMalloc.  This function
// runs the same two kernels — qkv_scatter (RMS norm across heads, RoPE, staging
// copy) and the tcgen05 attention — with the staging buffer taken from a
// fixed, file-scope device array instead, so the call itself allocates nothing.
//
// Contract.
//  * The caller passes every input and output as device pointers: qkv
//    [batch*seq, >= 3*heads*head_dim] bf16 (row stride qkv_stride elements), the
//    q/k RMS weights (bf16 [heads*head_dim]), the RoPE tables (fp32
//    [seq, head_dim/2], or null for no rotation), out [batch*seq, heads*head_dim]
//    bf16 (row stride out_stride), and optionally a device int[2] status word
//    that receives an error code if a bounded wait inside the kernels expires
//    (the caller zeroes it; null disables reporting).
//  * Supported shapes: head_dim 64 or 128 and heads*head_dim one of 512, 1024,
//    1536, 2048 or 3072 (the widths the norm/RoPE kernel is instantiated for);
//    anything else is DS_NOALLOC_BAD_ARGUMENT.
//  * Alignment: qkv, wq, wk, out, rope_cos and rope_sin must start on a 16-byte
//    boundary and both row strides must be multiples of 8 elements (16 bytes);
//    the kernels use 16-byte vector loads and stores, so a misaligned pointer
//    (an offset slice, say) is rejected with DS_NOALLOC_BAD_ARGUMENT up front.
//  * The staging buffer needs batch*seq*3*heads*head_dim*2 bytes and must fit
//    in kScratchBytes (16 MiB); larger problems are rejected with
//    DS_NOALLOC_TOO_LARGE before anything is launched.
//  * The array exists once per GPU that loads this library and stays reserved
//    until the process exits.  Every call on a device uses the same array and
//    leaves its contents behind; nothing in it has to start at zero (each call
//    overwrites the part it reads before reading it).  Two calls whose kernels
//    overlap on the GPU (different streams, or different host threads on the
//    same device) race on the array and produce garbage: serialise them.
//  * `stream` must belong to the current device (null: the legacy default
//    stream of the current device); a stream of another device is rejected with
//    DS_NOALLOC_BAD_ARGUMENT, since the array address is per device.
//  * The first call on each device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current) and caches it; that first
//    call should come before any stream capture on the device.
//  * Errors are attributed to this call: a CUDA error left pending by earlier,
//    unrelated work is cleared on entry, and each launch is checked on its own.
//  * No cudaMalloc, cudaFree or allocating library routine is called.
// Returns DS_NOALLOC_OK or one of the error codes in noalloc.h; kernels run on
// `stream` and are not synchronised.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <exception>
#include <mutex>

#include "kernels.h"
#include "noalloc.h"

namespace {

constexpr size_t kScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 64;

// Staging buffer of the allocation-free path (see the contract above).
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the array on the current device (looked up once per device).
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DS_NOALLOC_CUDA_ERROR;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return DS_NOALLOC_CUDA_ERROR;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return DS_NOALLOC_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool supported_width(long long width) {
  return width == 512 || width == 1024 || width == 1536 || width == 2048 || width == 3072;
}

}  // namespace

extern "C" int ds_fused_qkv_attention_noalloc(const void* qkv, long long qkv_stride, int batch, int seq, int heads,
                                              int head_dim, const void* wq, const void* wk, float eps,
                                              const float* rope_cos, const float* rope_sin, void* out,
                                              long long out_stride, int* status, void* stream) {
  if (qkv == nullptr || wq == nullptr || wk == nullptr || out == nullptr) return DS_NOALLOC_BAD_ARGUMENT;
  if (batch <= 0 || seq <= 0 || heads <= 0 || (head_dim != 64 && head_dim != 128)) return DS_NOALLOC_BAD_ARGUMENT;
  if ((rope_cos == nullptr) != (rope_sin == nullptr)) return DS_NOALLOC_BAD_ARGUMENT;
  const long long width = static_cast<long long>(heads) * head_dim;
  if (!supported_width(width) || qkv_stride < 3 * width || qkv_stride % 8 != 0 || out_stride < width ||
      out_stride % 8 != 0)
    return DS_NOALLOC_BAD_ARGUMENT;
  if (!aligned16(qkv) || !aligned16(wq) || !aligned16(wk) || !aligned16(out) ||
      (rope_cos != nullptr && (!aligned16(rope_cos) || !aligned16(rope_sin))))
    return DS_NOALLOC_BAD_ARGUMENT;
  const unsigned long long rows = static_cast<unsigned long long>(batch) * static_cast<unsigned long long>(seq);
  const unsigned long long need = rows * 3ull * static_cast<unsigned long long>(width) * 2ull;
  if (need > kScratchBytes) return DS_NOALLOC_TOO_LARGE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  (void)cudaGetLastError();  // a pending error of earlier, unrelated work is not this call's
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return DS_NOALLOC_CUDA_ERROR;
  if (s != nullptr) {
    int sdev = -1;
    if (cudaStreamGetDevice(s, &sdev) != cudaSuccess) return DS_NOALLOC_BAD_ARGUMENT;
    if (sdev != dev) return DS_NOALLOC_BAD_ARGUMENT;
  }
  void* scratch = nullptr;
  if (int rc = scratch_for_current_device(&scratch)) return rc;
  try {
    // 1) q/k RMS norm + RoPE; q, k, v staged as [rows, 3*width] in the scratch array
    ds::QkvScatterArgs sa;
    sa.qkv = qkv;
    sa.qkv_stride = qkv_stride;
    sa.rows = static_cast<int>(rows);
    sa.seq_local = seq;
    sa.heads = heads;
    sa.head_dim = head_dim;
    sa.wq = wq;
    sa.wk = wk;
    sa.eps = eps;
    sa.rope_cos = rope_cos;
    sa.rope_sin = rope_sin;
    sa.group.rank = 0;
    sa.group.size = 1;
    sa.group.base[0] = scratch;
    sa.recv_off = 0;
    ds::launch_qkv_scatter(sa, s);
    if (cudaGetLastError() != cudaSuccess) return DS_NOALLOC_LAUNCH_ERROR;
    // 2) attention reads the staged q/k/v and writes the caller's output
    const unsigned char* base = static_cast<const unsigned char*>(scratch);
    ds::AttnArgs aa;
    aa.q = base;
    aa.k = base + width * 2;
    aa.v = base + width * 4;
    aa.q_row_stride = aa.k_row_stride = aa.v_row_stride = 3 * width;
    aa.o = out;
    aa.o_row_stride = out_stride;
    aa.total_q = aa.total_k = static_cast<int>(rows);
    aa.batch = batch;
    aa.seq_q = aa.seq_k = seq;
    aa.heads = aa.heads_kv = heads;
    aa.head_dim = head_dim;
    aa.softmax_scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    aa.status = status;
    ds::launch_attention(aa, s);
    if (cudaGetLastError() != cudaSuccess) return DS_NOALLOC_LAUNCH_ERROR;
  } catch (const std::exception&) {
    // every argument the launchers check is checked above, so a throw here is a host-side
    // failure of the launch set-up (for example a tensor-map encode), not a bad argument
    return DS_NOALLOC_INTERNAL_ERROR;
  }
  return DS_NOALLOC_OK;
}
