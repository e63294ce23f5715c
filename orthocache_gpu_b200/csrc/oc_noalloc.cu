// Allocation-free entry point: oc_fused_attention_v2 with its split-K scratch
// in a statically reserved device array instead of a caller workspace.
//
// Some callers cannot allocate device memory at all (they run inside another
// framework's memory pool, under a fixed budget, or behind an interface that
// only passes inputs and outputs).  For them the library reserves
// kScratchBytes on every GPU that loads it; the reservation lasts until the
// process exits.  In host code `g_scratch` only names the array: its device
// address comes from cudaGetSymbolAddress, looked up once per device on the
// first call with that device current (so make the first call before any
// stream capture).  Every launch writes the parts of the array it later
// reads, so the array needs no clearing between calls; all calls share it,
// so calls that overlap on the GPU race.
#include <mutex>

#include "../../include/orthocache_b200.h"
#include "oc_dispatch.h"

namespace {

constexpr size_t kScratchBytes = size_t(2) << 20;  // 2 MiB per device
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {nullptr};

// Device address of g_scratch on the current device (looked up once).
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return OC_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_addr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_scratch) != cudaSuccess || ptr == nullptr) return OC_ERR_CUDA;
    g_addr[dev] = ptr;
  }
  *out = g_addr[dev];
  return OC_OK;
}

}  // namespace

extern "C" int oc_fused_attention_v2_noalloc(const void* q, int q_dtype, int64_t q_head_stride, const void* keys,
                                             int k_dtype, int64_t k_head_stride, int64_t k_tok_stride,
                                             const void* values, int v_dtype, int64_t v_head_stride,
                                             int64_t v_tok_stride, int num_heads, int64_t seq_len, int head_dim,
                                             double zeta_max, int num_splits, int num_sms, void* out,
                                             int out_dtype, int64_t out_head_stride, uint8_t* mask_out,
                                             uint32_t* retained, uint32_t* status, void* stream) {
  if (num_heads < 1 || seq_len < 0 || head_dim < 1) return OC_ERR_INVALID;
  // resolve the split count exactly as oc_fused_attention_v2 does, to size the scratch
  int sms = num_sms;
  if (sms <= 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms < 1) sms = 1;
  }
  const int64_t tiles = seq_len / 64;
  int splits = num_splits > 0 ? num_splits : oc_auto_num_splits(tiles, sms);
  if (tiles > 0 && splits > tiles) splits = (int)tiles;
  if (splits < 1) splits = 1;
  const size_t need = oc_workspace_bytes(num_heads, 1, tiles, head_dim);
  if (need > kScratchBytes) return OC_ERR_TOO_LARGE;
  void* ws = nullptr;
  const int r = scratch_address(&ws);
  if (r != OC_OK) return r;
  return oc_fused_attention_v2(q, q_dtype, q_head_stride, keys, k_dtype, k_head_stride, k_tok_stride, values,
                               v_dtype, v_head_stride, v_tok_stride, num_heads, seq_len, head_dim, zeta_max,
                               splits, sms, out, out_dtype, out_head_stride, mask_out, retained, status, ws,
                               kScratchBytes, stream);
}
