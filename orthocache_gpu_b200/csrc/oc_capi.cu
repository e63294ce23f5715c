// C ABI of liborthocache_b200.so: argument validation, the reference's
// threshold semantics, split selection, and dispatch to the kernel
// instantiations.  Declarations and contracts: include/orthocache_b200.h.
#include <cmath>
#include <cfloat>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <utility>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "../../include/orthocache_b200.h"
#include "oc_decode.cuh"
#include "oc_dispatch.h"

namespace {

using oc::DecodeParams;


int elem_bytes(int dt) {
  switch (dt) {
    case OC_F32: return 4;
    case OC_F16: case OC_BF16: return 2;
    case OC_F8E4M3: return 1;
    default: return 0;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Largest float32 <= x: the float threshold t with  (double)z > x  <=>  z > t
// and  (double)z <= x  <=>  z <= t  for every float32 z.
float round_down_f32(double x) {
  if (std::isnan(x)) return NAN;
  float f = static_cast<float>(x);
  if (static_cast<double>(f) > x) f = std::nextafterf(f, -INFINITY);
  return f;
}

int gc_for_group(int group) {
  if (group <= 1) return 1;
  if (group <= 2) return 2;
  if (group <= 4) return 4;
  return 8;
}

bool hd_supported(int hd, int k_dtype) {
  if (hd != 16 && hd != 32 && hd != 64 && hd != 128 && hd != 256) return false;
  if (k_dtype == OC_F32 && hd > 128) return false;
  return true;
}

bool types_supported(int q_dtype, int k_dtype, int v_dtype, int out_dtype) {
  auto qv = [](int d) { return d == OC_F32 || d == OC_F16 || d == OC_BF16; };
  if (!qv(q_dtype) || !qv(out_dtype) || !qv(v_dtype)) return false;
  if (k_dtype == OC_F8E4M3) return true;
  return k_dtype == v_dtype;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// TMA descriptor of the K or V tensor as a 4-D view {head_dim, token, kv
// head, sequence-or-block} whose dimensions 1..3 are ordered by stride (the
// copy engine wants increasing strides); pos[role] returns the dimension of
// role 0 (token), 1 (kv head), 2 (sequence or block).  Box: one 64-column
// panel with the 128-byte swizzle (tensor-core path) or a whole row, by
// p.box_rows tokens.
bool make_map(CUtensorMap* m, const char* base, int dtype, int hd, bool tc, const DecodeParams& p, bool isv,
              int (&pos)[3]) {
  const auto enc = tensor_map_encoder();
  if (!enc) return false;
  const int esz = elem_bytes(dtype);
  int64_t size[3], stride[3];
  size[0] = p.layout == oc::LAYOUT_LINEAR ? (int64_t)p.num_tiles * 64 : ((int64_t)1 << p.block_shift);
  stride[0] = isv ? p.v_tok_stride : p.k_tok_stride;
  size[1] = p.num_kv_heads;
  stride[1] = isv ? p.v_head_stride : p.k_head_stride;
  size[2] = p.layout == oc::LAYOUT_LINEAR ? p.num_seqs : p.num_blocks;
  stride[2] = p.layout == oc::LAYOUT_LINEAR ? (isv ? p.v_seq_stride : p.k_seq_stride)
                                            : (isv ? p.v_blk_stride : p.k_blk_stride);
  // order the roles by stride; extent-1 roles go last with a stride that nests
  int order[3] = {0, 1, 2};
  auto key = [&](int r) { return size[r] == 1 ? INT64_MAX : stride[r]; };
  for (int i = 0; i < 3; ++i)
    for (int j = i + 1; j < 3; ++j)
      if (key(order[j]) < key(order[i])) std::swap(order[i], order[j]);
  cuuint64_t gdim[4], gstr[3];
  gdim[0] = (cuuint64_t)hd;
  int64_t last = (int64_t)hd * esz;
  for (int i = 0; i < 3; ++i) {
    const int r = order[i];
    gdim[i + 1] = (cuuint64_t)size[r];
    int64_t st = stride[r];
    if (size[r] == 1 || st <= 0) st = (last + 15) / 16 * 16;
    gstr[i] = (cuuint64_t)st;
    last = st * size[r];
    pos[r] = i + 1;
  }
  cuuint32_t box[4] = {(cuuint32_t)(tc ? oc::kTcPanel : hd), 1, 1, 1};
  box[pos[0]] = (cuuint32_t)p.box_rows;
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUtensorMapDataType dt;
  switch (dtype) {
    case OC_F32: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; break;
    case OC_F16: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; break;
    case OC_BF16: dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; break;
    default: dt = CU_TENSOR_MAP_DATA_TYPE_UINT8; break;
  }
  const CUresult r = enc(m, dt, 4, const_cast<char*>(base), gdim, gstr, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         tc ? (oc::kTcPanel == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B)
                            : CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

unsigned long long* g_trace = nullptr;  // diagnostics buffer (oc_debug_set_trace)

// Encoded tensor maps are pure functions of their inputs; decode calls repeat
// them (same cache, same shapes), so each host thread keeps the last few.
struct MapKey {
  const char* base;
  int dtype, hd, tc, isv, layout, box_rows, block_shift, num_kv_heads, num_seqs, num_blocks, num_tiles;
  int64_t s_tok, s_head, s_outer;
  bool operator==(const MapKey& o) const { return std::memcmp(this, &o, sizeof(MapKey)) == 0; }
};
struct MapEntry {
  MapKey key;
  CUtensorMap map;
  int pos[3];
  bool used;
};

bool cached_map(CUtensorMap* m, const char* base, int dtype, int hd, bool tc, const DecodeParams& p, bool isv,
                int (&pos)[3]) {
  thread_local MapEntry cache[8] = {};
  thread_local unsigned next = 0;
  MapKey k;
  std::memset(&k, 0, sizeof(k));  // padding bytes take part in the comparison
  k.base = base;
  k.dtype = dtype;
  k.hd = hd;
  k.tc = tc;
  k.isv = isv;
  k.layout = p.layout;
  k.box_rows = p.box_rows;
  k.block_shift = p.block_shift;
  k.num_kv_heads = p.num_kv_heads;
  k.num_seqs = p.num_seqs;
  k.num_blocks = p.num_blocks;
  k.num_tiles = p.num_tiles;
  k.s_tok = isv ? p.v_tok_stride : p.k_tok_stride;
  k.s_head = isv ? p.v_head_stride : p.k_head_stride;
  k.s_outer = p.layout == oc::LAYOUT_LINEAR ? (isv ? p.v_seq_stride : p.k_seq_stride)
                                            : (isv ? p.v_blk_stride : p.k_blk_stride);
  for (auto& e : cache)
    if (e.used && e.key == k) {
      *m = e.map;
      for (int i = 0; i < 3; ++i) pos[i] = e.pos[i];
      return true;
    }
  if (!make_map(m, base, dtype, hd, tc, p, isv, pos)) return false;
  MapEntry& e = cache[next++ % 8];
  e.key = k;
  e.map = *m;
  for (int i = 0; i < 3; ++i) e.pos[i] = pos[i];
  e.used = true;
  return true;
}

int run(const DecodeParams& p0, int k_dtype, int v_dtype, int hd, bool attn, int sms, cudaStream_t st) {
  DecodeParams p = p0;
  p.trace = g_trace;
  const int gc = gc_for_group(p.group);
  p.box_rows = p.layout == oc::LAYOUT_LINEAR ? 64 : ((1 << p.block_shift) < 64 ? (1 << p.block_shift) : 64);
  // tensor cores need 16-bit keys, values of the same type and, for attention,
  // queries of that type too (the logits are then exact products in fp32);
  // swizzled boxes start on 1024-byte boundaries, so at least 8 rows a box
  // (queries are read as 32-bit pairs there: 4-byte aligned rows)
  const bool q_pairs = (reinterpret_cast<uintptr_t>(p.q) & 3u) == 0 && (p.q_seq_stride & 1) == 0 &&
                       (p.q_head_stride & 1) == 0;
  const bool tc = (k_dtype == OC_F16 || k_dtype == OC_BF16) && v_dtype == k_dtype && hd >= 64 &&
                  (!attn || (p.q_dtype == k_dtype && q_pairs)) && p.box_rows >= 8;
  // unswizzled boxes start on 128-byte boundaries
  if (!tc && ((p.box_rows * hd * elem_bytes(k_dtype)) % 128 || (attn && (p.box_rows * hd * elem_bytes(v_dtype)) % 128)))
    return OC_ERR_UNSUPPORTED;
  oc::TensorMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  const bool any_tile = p.num_tiles > 0 && p.k != nullptr;
  if (any_tile) {
    if (!cached_map(&maps.k, p.k, k_dtype, hd, tc, p, false, p.tm_pos_k)) return OC_ERR_INVALID;
    if (attn && !cached_map(&maps.v, p.v, v_dtype, hd, tc, p, true, p.tm_pos_v)) return OC_ERR_INVALID;
  } else {
    for (int i = 0; i < 3; ++i) p.tm_pos_k[i] = p.tm_pos_v[i] = i + 1;
  }
#define OC_HDS(K, ...)                                              \
  switch (hd) {                                                     \
    case 16: return oc::dispatch_##K##_16(p, maps, v_dtype, gc, attn, sms, st, tc);   \
    case 32: return oc::dispatch_##K##_32(p, maps, v_dtype, gc, attn, sms, st, tc);   \
    case 64: return oc::dispatch_##K##_64(p, maps, v_dtype, gc, attn, sms, st, tc);   \
    case 128: return oc::dispatch_##K##_128(p, maps, v_dtype, gc, attn, sms, st, tc); \
    __VA_ARGS__                                                     \
    default: return OC_ERR_UNSUPPORTED;                             \
  }
  switch (k_dtype) {
    case OC_F32: OC_HDS(f32)
    case OC_F16: OC_HDS(f16, case 256: return oc::dispatch_f16_256(p, maps, v_dtype, gc, attn, sms, st, tc);)
    case OC_BF16: OC_HDS(bf16, case 256: return oc::dispatch_bf16_256(p, maps, v_dtype, gc, attn, sms, st, tc);)
    case OC_F8E4M3: OC_HDS(f8, case 256: return oc::dispatch_f8_256(p, maps, v_dtype, gc, attn, sms, st, tc);)
    default: return OC_ERR_UNSUPPORTED;
  }
#undef OC_HDS
}

int sms_or_device(int num_sms) {
  if (num_sms > 0) return num_sms;
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 1;
}

// Workspace layout (every region 256-byte aligned):
//   fixed header (kFixedBytes): the per-unit tile prefix for the merge
//     kernel and the per-team retained-tile counts (both written by every
//     launch before they are read, so the workspace needs no initialisation)
//   part  partial states, 2 slots per team of warps: 2*kMaxTeams*gc*(hd+32) f32
//         (each of a team's P panels keeps its columns plus m, l and padding)
constexpr int64_t kMaxUnits = 2048;  // units per launch (shared-memory prefix arrays)
constexpr int64_t kMaxTeams = 1280;  // teams of warps per grid (the kernel clamps its grid to this)
constexpr size_t pad256(size_t b) { return (b + 255) & ~size_t(255); }
constexpr size_t kFixedBytes = pad256(4 * 4 * kMaxUnits);
// per-team retained-tile counts live in the second half of the fixed header
constexpr size_t kTeamKeptOffset = pad256(4 * (kMaxUnits + 1));
static_assert(kTeamKeptOffset + 4 * kMaxTeams <= kFixedBytes, "fixed workspace header");

struct WsLayout {
  size_t part, total;
};

WsLayout ws_layout(int64_t /*units*/, int gc, int64_t /*num_tiles*/, int hd) {
  WsLayout L;
  L.part = kFixedBytes;
  L.total = L.part + pad256(4 * (size_t)2 * kMaxTeams * gc * (hd + 32));
  return L;
}

int attach_workspace(DecodeParams& p, int64_t units, int hd, void* ws, size_t ws_bytes) {
  const int gc = gc_for_group(p.group);
  const WsLayout L = ws_layout(units, gc, p.num_tiles, hd);
  if (ws == nullptr || ws_bytes < L.total || !aligned16(ws)) return OC_ERR_WORKSPACE;
  char* b = static_cast<char*>(ws);
  p.tile_prefix = reinterpret_cast<int*>(b);
  p.team_kept = reinterpret_cast<int*>(b + kTeamKeptOffset);
  p.part = reinterpret_cast<float*>(b + L.part);
  return OC_OK;
}

DecodeParams blank() {
  DecodeParams p;
  std::memset(&p, 0, sizeof(p));
  p.layout = oc::LAYOUT_LINEAR;
  p.k_deq_dtype = -1;
  p.k_deq_scale = 1.f;
  p.block_shift = 0;
  p.num_seqs = 1;
  p.group = 1;
  return p;
}

bool stride_ok(int64_t stride_elems, int esz) { return ((stride_elems * esz) & 15) == 0; }

}  // namespace

extern "C" {

const char* oc_status_string(int code) {
  switch (code) {
    case OC_OK: return "ok";
    case OC_ERR_INVALID: return "invalid argument (pointer, size, stride or 16-byte alignment)";
    case OC_ERR_UNSUPPORTED: return "unsupported dtype / head_dim combination";
    case OC_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case OC_ERR_CUDA: return "CUDA launch failed";
    case OC_ERR_TOO_LARGE:
      return "problem needs more scratch than the fixed 2 MiB of oc_fused_attention_v2_noalloc";
    default: return "unknown status";
  }
}

int oc_version(void) { return 100; }

void oc_debug_set_trace(void* buffer) { g_trace = static_cast<unsigned long long*>(buffer); }

size_t oc_workspace_bytes(int64_t num_groups, int group, int64_t num_tiles, int head_dim) {
  if (num_groups < 1 || group < 1 || num_tiles < 0 || head_dim < 1) return 0;
  const int gc = gc_for_group(group);
  int64_t units = num_groups * ((group + gc - 1) / gc);
  if (units > kMaxUnits) units = kMaxUnits;  // larger batches run as several launches
  return ws_layout(units, gc, num_tiles, head_dim).total;
}

int oc_auto_num_splits(int64_t num_tiles, int num_sms) {
  int64_t max_splits = num_tiles / 4;
  if (max_splits < 1) max_splits = 1;
  int64_t s = num_sms;
  if (max_splits < s) s = max_splits;
  if (num_tiles < s) s = num_tiles;
  return s < 1 ? 1 : (int)s;
}

int oc_fwht_eviction(const void* keys, int k_dtype, int64_t num_tokens, int head_dim, int64_t k_tok_stride,
                     double zeta_max, uint8_t* mask_out, float* zeta_out, uint32_t* status, void* stream) {
  const int kb = elem_bytes(k_dtype);
  if (!keys || !mask_out || !status || kb == 0 || num_tokens < 0 || (num_tokens % 64) != 0)
    return OC_ERR_INVALID;
  if (!hd_supported(head_dim, k_dtype)) return OC_ERR_UNSUPPORTED;
  if (!aligned16(keys) || !stride_ok(k_tok_stride, kb)) return OC_ERR_INVALID;
  const int64_t tiles = num_tokens / 64;
  if (tiles == 0) return OC_OK;
  DecodeParams p = blank();
  p.k = static_cast<const char*>(keys);
  p.k_tok_stride = k_tok_stride * kb;
  p.num_kv_heads = 1;
  p.num_tiles = (int)tiles;
  p.num_splits = oc_auto_num_splits(tiles, sms_or_device(0));
  p.gate = oc::GATE_ZETA_MASK;
  p.thr = static_cast<float>(zeta_max);  // torch compares a float32 tensor with the scalar in float32
  p.mask = reinterpret_cast<int8_t*>(mask_out);
  p.score = zeta_out;
  p.status = status;
  return run(p, k_dtype, k_dtype, head_dim, false, sms_or_device(0), static_cast<cudaStream_t>(stream));
}

static int v3_common(DecodeParams& p, const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
                     const void* keys, int k_dtype, int64_t k_seq_stride, int64_t k_head_stride,
                     int64_t k_tok_stride, const void* values, int v_dtype, int64_t v_seq_stride,
                     int64_t v_head_stride, int64_t v_tok_stride, int num_seqs, int num_kv_heads, int group,
                     int64_t seq_len, int head_dim, int num_splits, int num_sms, void* out, int out_dtype,
                     int64_t out_seq_stride, int64_t out_head_stride, uint8_t* mask_out, uint32_t* retained,
                     uint32_t* status, void* workspace, size_t workspace_bytes, void* stream) {
  const int kb = elem_bytes(k_dtype), vb = elem_bytes(v_dtype);
  if (!q || !status || kb == 0 || vb == 0) return OC_ERR_INVALID;
  if (seq_len > 0 && (!keys || !values)) return OC_ERR_INVALID;
  if (num_seqs < 1 || num_kv_heads < 1 || group < 1 || seq_len < 0 || (seq_len % 64) != 0) return OC_ERR_INVALID;
  if (!types_supported(q_dtype, k_dtype, v_dtype, out_dtype) || !hd_supported(head_dim, k_dtype))
    return OC_ERR_UNSUPPORTED;
  if (!aligned16(keys) || !aligned16(values)) return OC_ERR_INVALID;  // null is aligned
  if (!stride_ok(k_tok_stride, kb) || !stride_ok(v_tok_stride, vb) || !stride_ok(k_head_stride, kb) ||
      !stride_ok(v_head_stride, vb) || !stride_ok(k_seq_stride, kb) || !stride_ok(v_seq_stride, vb))
    return OC_ERR_INVALID;
  const int64_t tiles = seq_len / 64;
  if (tiles > INT32_MAX / 64) return OC_ERR_INVALID;
  p.q = q;
  p.q_dtype = q_dtype;
  p.q_seq_stride = q_seq_stride;
  p.q_head_stride = q_head_stride;
  p.k = static_cast<const char*>(keys);
  p.v = static_cast<const char*>(values);
  p.k_seq_stride = k_seq_stride * kb;
  p.k_head_stride = k_head_stride * kb;
  p.k_tok_stride = k_tok_stride * kb;
  p.v_seq_stride = v_seq_stride * vb;
  p.v_head_stride = v_head_stride * vb;
  p.v_tok_stride = v_tok_stride * vb;
  p.num_seqs = num_seqs;
  p.num_kv_heads = num_kv_heads;
  p.group = group;
  p.num_tiles = (int)tiles;
  p.num_splits = num_splits > 0 ? num_splits : oc_auto_num_splits(tiles, sms_or_device(num_sms));
  if (tiles > 0 && p.num_splits > tiles) p.num_splits = (int)tiles;
  if (p.num_splits < 1) p.num_splits = 1;
  if (p.num_splits > 65535) return OC_ERR_INVALID;
  p.scale_log2 = static_cast<float>((1.0 / std::sqrt((double)head_dim)) * 1.4426950408889634);
  p.out = out;
  p.out_dtype = out_dtype;
  p.out_seq_stride = out_seq_stride;
  p.out_head_stride = out_head_stride;
  p.mask = reinterpret_cast<int8_t*>(mask_out);
  p.stats = retained;
  p.status = status;
  if (p.sh_acc == nullptr && out == nullptr) return OC_ERR_INVALID;
  const int sms = sms_or_device(num_sms);
  const int gc = gc_for_group(group);
  const int64_t units_per_seq = (int64_t)num_kv_heads * ((group + gc - 1) / gc);
  if (units_per_seq > kMaxUnits) return OC_ERR_INVALID;
  // the kernel keeps per-unit prefix arrays in shared memory: batches of at
  // most kMaxUnits units run as consecutive launches on the stream
  const int64_t seqs_per_launch = kMaxUnits / units_per_seq;
  const int qsz = elem_bytes(q_dtype), osz = elem_bytes(out_dtype);
  for (int64_t s0 = 0; s0 < num_seqs; s0 += seqs_per_launch) {
    DecodeParams pc = p;
    const int64_t ns = (num_seqs - s0) < seqs_per_launch ? (num_seqs - s0) : seqs_per_launch;
    pc.num_seqs = (int)ns;
    pc.q = static_cast<const char*>(q) + s0 * q_seq_stride * qsz;
    if (p.layout == oc::LAYOUT_LINEAR) {
      if (pc.k) pc.k += s0 * p.k_seq_stride;
      if (pc.v) pc.v += s0 * p.v_seq_stride;
    } else {
      pc.block_tables = p.block_tables + s0 * p.bt_seq_stride;
      if (p.seq_lens) pc.seq_lens = p.seq_lens + s0;
    }
    if (out) pc.out = static_cast<char*>(out) + s0 * out_seq_stride * osz;
    if (p.sh_acc) {  // merged states are indexed by (sequence, query head) inside a launch
      const int64_t u0 = s0 * num_kv_heads * group;
      pc.sh_m = p.sh_m + u0;
      pc.sh_l = p.sh_l + u0;
      pc.sh_acc = p.sh_acc + u0 * out_head_stride;
    }
    if (p.mask) pc.mask = p.mask + s0 * num_kv_heads * tiles;
    pc.stats_add = s0 > 0 ? 1 : 0;  // the first launch sets the count, later ones add
    if (p.tile_list) {
      pc.tile_list = p.tile_list + s0 * num_kv_heads * p.list_stride;
      pc.list_count = p.list_count + s0 * num_kv_heads;
    }
    const int r = attach_workspace(pc, ns * units_per_seq, head_dim, workspace, workspace_bytes);
    if (r != OC_OK) return r;
    const int e = run(pc, k_dtype, v_dtype, head_dim, true, sms, static_cast<cudaStream_t>(stream));
    if (e != OC_OK) return e;
  }
  return OC_OK;
}

int oc_fused_attention_v2(const void* q, int q_dtype, int64_t q_head_stride, const void* keys, int k_dtype,
                          int64_t k_head_stride, int64_t k_tok_stride, const void* values, int v_dtype,
                          int64_t v_head_stride, int64_t v_tok_stride, int num_heads, int64_t seq_len,
                          int head_dim, double zeta_max, int num_splits, int num_sms, void* out, int out_dtype,
                          int64_t out_head_stride, uint8_t* mask_out, uint32_t* retained, uint32_t* status,
                          void* workspace, size_t workspace_bytes, void* stream) {
  DecodeParams p = blank();
  p.gate = oc::GATE_ZETA_ATTN;
  p.thr = round_down_f32(zeta_max);
  // V2 is the kv_heads = num_heads, group = 1 case of the generic decode
  return v3_common(p, q, q_dtype, 0, q_head_stride, keys, k_dtype, 0, k_head_stride, k_tok_stride, values,
                   v_dtype, 0, v_head_stride, v_tok_stride, 1, num_heads, 1, seq_len, head_dim, num_splits,
                   num_sms, out, out_dtype, 0, out_head_stride, mask_out, retained, status, workspace,
                   workspace_bytes, stream);
}

int oc_fused_attention_v1(const void* q, int q_dtype, const void* keys, int k_dtype, int64_t k_tok_stride,
                          const void* values, int v_dtype, int64_t v_tok_stride, int64_t seq_len, int head_dim,
                          double zeta_max, int num_sms, void* out, int out_dtype, uint8_t* mask_out,
                          uint32_t* retained, uint32_t* status, void* workspace, size_t workspace_bytes,
                          void* stream) {
  return oc_fused_attention_v2(q, q_dtype, head_dim, keys, k_dtype, 0, k_tok_stride, values, v_dtype, 0,
                               v_tok_stride, 1, seq_len, head_dim, zeta_max, 0, num_sms, out, out_dtype,
                               head_dim, mask_out, retained, status, workspace, workspace_bytes, stream);
}

int oc_fused_attention_v3_gqa(const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
                              const void* keys, int k_dtype, int64_t k_seq_stride, int64_t k_head_stride,
                              int64_t k_tok_stride, const void* values, int v_dtype, int64_t v_seq_stride,
                              int64_t v_head_stride, int64_t v_tok_stride, int num_seqs, int num_kv_heads,
                              int group, int64_t seq_len, int head_dim, double tau, int num_splits, int num_sms,
                              void* out, int out_dtype, int64_t out_seq_stride, int64_t out_head_stride,
                              uint8_t* mask_out, uint32_t* retained, uint32_t* status, void* workspace,
                              size_t workspace_bytes, void* stream) {
  DecodeParams p = blank();
  p.gate = oc::GATE_CS;
  p.thr = round_down_f32(tau);
  return v3_common(p, q, q_dtype, q_seq_stride, q_head_stride, keys, k_dtype, k_seq_stride, k_head_stride,
                   k_tok_stride, values, v_dtype, v_seq_stride, v_head_stride, v_tok_stride, num_seqs,
                   num_kv_heads, group, seq_len, head_dim, num_splits, num_sms, out, out_dtype, out_seq_stride,
                   out_head_stride, mask_out, retained, status, workspace, workspace_bytes, stream);
}

int oc_fused_attention_v3_shard(const void* q, int q_dtype, int64_t q_head_stride, const void* keys, int k_dtype,
                                int64_t k_head_stride, int64_t k_tok_stride, const void* values, int v_dtype,
                                int64_t v_head_stride, int64_t v_tok_stride, int num_kv_heads, int group,
                                int64_t seq_len, int head_dim, double tau, int num_splits, int num_sms,
                                float* m_out, float* l_out, float* acc_out, uint8_t* mask_out,
                                const int32_t* seq_len_dev, uint32_t* retained, uint32_t* status,
                                void* workspace, size_t workspace_bytes, void* stream) {
  if (!m_out || !l_out || !acc_out) return OC_ERR_INVALID;
  DecodeParams p = blank();
  p.seq_lens = seq_len_dev;  // nullable: tokens actually decoded, read on the device
  p.gate = oc::GATE_CS;
  p.thr = round_down_f32(tau);
  p.sh_m = m_out;
  p.sh_l = l_out;
  p.sh_acc = acc_out;
  return v3_common(p, q, q_dtype, 0, q_head_stride, keys, k_dtype, 0, k_head_stride, k_tok_stride, values,
                   v_dtype, 0, v_head_stride, v_tok_stride, 1, num_kv_heads, group, seq_len, head_dim,
                   num_splits, num_sms, nullptr, OC_F32, 0, head_dim, mask_out, retained, status, workspace,
                   workspace_bytes, stream);
}

int oc_fused_attention_paged(const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
                             const void* k_cache, int k_dtype, int64_t k_blk_stride, int64_t k_head_stride,
                             int64_t k_tok_stride, const void* v_cache, int v_dtype, int64_t v_blk_stride,
                             int64_t v_head_stride, int64_t v_tok_stride, int num_blocks, int block_size,
                             const int32_t* block_tables, int64_t bt_seq_stride, int max_blocks,
                             const int32_t* seq_lens, int num_seqs, int num_kv_heads, int group, int head_dim,
                             int gate, double threshold, double k_scale, int num_splits, int num_sms, void* out,
                             int out_dtype,
                             int64_t out_seq_stride, int64_t out_head_stride, uint8_t* mask_out,
                             uint32_t* retained, uint32_t* status, void* workspace, size_t workspace_bytes,
                             void* stream) {
  if (!block_tables || block_size < 1 || (block_size & (block_size - 1)) || max_blocks < 0 || num_blocks < 1)
    return OC_ERR_INVALID;
  const int kb = elem_bytes(k_dtype), vb = elem_bytes(v_dtype);
  if (kb == 0 || vb == 0) return OC_ERR_INVALID;
  if (!stride_ok(k_blk_stride, kb) || !stride_ok(v_blk_stride, vb)) return OC_ERR_INVALID;
  const int64_t tokens = (int64_t)max_blocks * block_size;
  DecodeParams p = blank();
  if (gate == OC_GATE_ZETA) {
    p.gate = oc::GATE_ZETA_ATTN;
  } else if (gate == OC_GATE_CAUCHY_SCHWARZ) {
    p.gate = oc::GATE_CS;
  } else {
    return OC_ERR_INVALID;
  }
  p.thr = round_down_f32(threshold);
  if (k_dtype == OC_F8E4M3) {  // de-quantised into q's dtype, as the reference's paged path does
    if (q_dtype != OC_F32 && q_dtype != OC_F16 && q_dtype != OC_BF16) return OC_ERR_UNSUPPORTED;
    p.k_deq_dtype = q_dtype;  // OC_F32/F16/BF16 equal oc::DT_F32/F16/BF16
    p.k_deq_scale = static_cast<float>(k_scale);
  }
  p.layout = oc::LAYOUT_PAGED;
  p.block_tables = block_tables;
  p.bt_seq_stride = bt_seq_stride;
  p.k_blk_stride = k_blk_stride * kb;
  p.v_blk_stride = v_blk_stride * vb;
  int shift = 0;
  while ((1 << shift) < block_size) ++shift;
  p.block_shift = shift;
  p.num_blocks = num_blocks;
  p.seq_lens = seq_lens;
  // the paged grid covers floor(max_blocks*block_size / 64) tiles per sequence
  const int64_t seq_len = tokens - tokens % 64;
  // tiles of a unit are processed in sequence order (one split), so that each
  // team's copies walk the block table forward and read it in windows;
  // num_splits is accepted for compatibility and does not change the result
  (void)num_splits;
  return v3_common(p, q, q_dtype, q_seq_stride, q_head_stride, k_cache, k_dtype, 0, k_head_stride, k_tok_stride,
                   v_cache, v_dtype, 0, v_head_stride, v_tok_stride, num_seqs, num_kv_heads, group, seq_len,
                   head_dim, 1, num_sms, out, out_dtype, out_seq_stride, out_head_stride, mask_out,
                   retained, status, workspace, workspace_bytes, stream);
}

namespace {
// bytes after the regular workspace: per-(sequence, kv head) counts, then the tile lists
size_t cached_extra(int64_t groups, int64_t tiles) { return pad256(4 * (size_t)groups) + pad256(4 * (size_t)groups * tiles); }
}  // namespace

size_t oc_cached_workspace_bytes(int64_t num_groups, int group, int64_t num_tiles, int head_dim) {
  const size_t b = oc_workspace_bytes(num_groups, group, num_tiles, head_dim);
  return b == 0 ? 0 : b + cached_extra(num_groups, num_tiles);
}

int oc_tile_high_norms(const void* keys, int k_dtype, int num_heads, int64_t num_tokens, int head_dim,
                       int64_t k_head_stride, int64_t k_tok_stride, int high_start, int high_end, float* out,
                       int64_t out_head_stride, void* stream) {
  if (!keys || !out || num_heads < 0 || num_tokens < 0 || (num_tokens % 64) != 0) return OC_ERR_INVALID;
  if (elem_bytes(k_dtype) == 0) return OC_ERR_UNSUPPORTED;
  if (head_dim < 1 || head_dim > 256) return OC_ERR_UNSUPPORTED;
  if (high_start < 0 || high_end > 64 || high_start > high_end) return OC_ERR_INVALID;
  if (num_tokens / 64 > INT32_MAX) return OC_ERR_INVALID;
  return oc::launch_tile_high_norms(keys, k_dtype, num_heads, (int)(num_tokens / 64), head_dim, k_head_stride,
                                    k_tok_stride, high_start, high_end, out, out_head_stride,
                                    static_cast<cudaStream_t>(stream));
}

static float gate_threshold(double tau, int head_dim) {
  // torch compares the float32 bounds with the Python scalar tau * (64 * head_dim) cast to float32
  return static_cast<float>(tau * (64.0 * head_dim));
}

int oc_decode_gate(const void* q, int q_dtype, int64_t q_head_stride, int num_kv_heads, int group, int head_dim,
                   const float* norms, int64_t norm_head_stride, int num_tiles, int max_tiles, double tau,
                   int tight, int low_band, int q_stat, uint8_t* evict_out, float* q_norms_out, void* stream) {
  if (!q || !norms || num_kv_heads < 1 || group < 1 || group > 64 || head_dim < 1 || num_tiles < 0 ||
      max_tiles < num_tiles || low_band < 1 || low_band > 32 || (tight && head_dim % low_band))
    return OC_ERR_INVALID;
  if (q_dtype != OC_F32 && q_dtype != OC_F16 && q_dtype != OC_BF16) return OC_ERR_UNSUPPORTED;
  oc::GateArgs a{};
  a.q = q;
  a.q_dtype = q_dtype;
  a.q_head_stride = q_head_stride;
  a.num_seqs = 1;
  a.num_kv_heads = num_kv_heads;
  a.group = group;
  a.head_dim = head_dim;
  a.norms = norms;
  a.norm_head_stride = norm_head_stride;
  a.num_tiles = num_tiles;
  a.max_tiles = max_tiles;
  a.thr = gate_threshold(tau, head_dim);
  a.tight = tight;
  a.low_band = low_band;
  a.stat_median = q_stat;
  a.evict = evict_out;
  a.evict_stride = max_tiles;
  a.q_norms = q_norms_out;
  return oc::launch_decode_gate(a, static_cast<cudaStream_t>(stream));
}

int oc_fused_attention_cached(const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
                              const void* keys, int k_dtype, int64_t k_seq_stride, int64_t k_head_stride,
                              int64_t k_tok_stride, const void* values, int v_dtype, int64_t v_seq_stride,
                              int64_t v_head_stride, int64_t v_tok_stride, int num_seqs, int num_kv_heads,
                              int group, int64_t seq_len, int head_dim, const float* norms,
                              int64_t norm_seq_stride, int64_t norm_head_stride, double tau, int tight,
                              int q_stat, int num_sms, void* out, int out_dtype, int64_t out_seq_stride,
                              int64_t out_head_stride, float* m_out, float* l_out, float* acc_out,
                              uint8_t* evict_out, float* q_norms_out, uint32_t* retained, uint32_t* status,
                              void* workspace, size_t workspace_bytes, void* stream) {
  if ((acc_out != nullptr) != (m_out != nullptr) || (acc_out != nullptr) != (l_out != nullptr)) return OC_ERR_INVALID;
  if (!norms || num_seqs < 1 || num_kv_heads < 1 || group < 1 || group > 64 || seq_len < 0 || (seq_len % 64))
    return OC_ERR_INVALID;
  if (tight && head_dim % 8) return OC_ERR_INVALID;
  const int64_t tiles = seq_len / 64;
  const int64_t groups = (int64_t)num_seqs * num_kv_heads;
  const size_t base = oc_workspace_bytes(groups, group, tiles, head_dim);
  if (!workspace || base == 0 || workspace_bytes < base + cached_extra(groups, tiles)) return OC_ERR_WORKSPACE;
  int* count = reinterpret_cast<int*>(static_cast<char*>(workspace) + base);
  int* list = reinterpret_cast<int*>(static_cast<char*>(workspace) + base + pad256(4 * (size_t)groups));
  if (q_dtype != OC_F32 && q_dtype != OC_F16 && q_dtype != OC_BF16) return OC_ERR_UNSUPPORTED;
  oc::GateArgs a{};
  a.q = q;
  a.q_dtype = q_dtype;
  a.q_seq_stride = q_seq_stride;
  a.q_head_stride = q_head_stride;
  a.num_seqs = num_seqs;
  a.num_kv_heads = num_kv_heads;
  a.group = group;
  a.head_dim = head_dim;
  a.norms = norms;
  a.norm_seq_stride = norm_seq_stride;
  a.norm_head_stride = norm_head_stride;
  a.num_tiles = (int)tiles;
  a.max_tiles = (int)tiles;
  a.thr = gate_threshold(tau, head_dim);
  a.tight = tight;
  a.low_band = 8;
  a.stat_median = q_stat;
  a.evict = evict_out;
  a.evict_stride = tiles;
  a.q_norms = q_norms_out;
  a.list = list;
  a.list_stride = tiles;
  a.count = count;
  const int g = oc::launch_decode_gate(a, static_cast<cudaStream_t>(stream));
  if (g != OC_OK) return g;
  DecodeParams p = blank();
  p.gate = oc::GATE_LIST;
  p.tile_list = list;
  p.list_count = count;
  p.list_stride = tiles;
  if (acc_out) {  // merged softmax states (m in log2 units, l, unnormalised acc) instead of the output
    p.sh_m = m_out;
    p.sh_l = l_out;
    p.sh_acc = acc_out;
    return v3_common(p, q, q_dtype, q_seq_stride, q_head_stride, keys, k_dtype, k_seq_stride, k_head_stride,
                     k_tok_stride, values, v_dtype, v_seq_stride, v_head_stride, v_tok_stride, num_seqs,
                     num_kv_heads, group, seq_len, head_dim, 1, num_sms, nullptr, OC_F32, 0, head_dim, nullptr,
                     retained, status, workspace, base, stream);
  }
  return v3_common(p, q, q_dtype, q_seq_stride, q_head_stride, keys, k_dtype, k_seq_stride, k_head_stride,
                   k_tok_stride, values, v_dtype, v_seq_stride, v_head_stride, v_tok_stride, num_seqs,
                   num_kv_heads, group, seq_len, head_dim, 1, num_sms, out, out_dtype, out_seq_stride,
                   out_head_stride, nullptr, retained, status, workspace, base, stream);
}

int oc_fused_attention_tiles(const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
                             const void* keys, int k_dtype, int64_t k_seq_stride, int64_t k_head_stride,
                             int64_t k_tok_stride, const void* values, int v_dtype, int64_t v_seq_stride,
                             int64_t v_head_stride, int64_t v_tok_stride, int num_seqs, int num_kv_heads,
                             int group, int64_t seq_len, int head_dim, const int32_t* tile_list,
                             int64_t list_stride, const int32_t* list_count, int num_sms, void* out, int out_dtype,
                             int64_t out_seq_stride, int64_t out_head_stride, float* m_out, float* l_out,
                             float* acc_out, uint32_t* retained, uint32_t* status, void* workspace,
                             size_t workspace_bytes, void* stream) {
  if (!tile_list || !list_count || list_stride < 0) return OC_ERR_INVALID;
  if ((acc_out != nullptr) != (m_out != nullptr) || (acc_out != nullptr) != (l_out != nullptr)) return OC_ERR_INVALID;
  DecodeParams p = blank();
  p.gate = oc::GATE_LIST;
  p.tile_list = tile_list;
  p.list_count = list_count;
  p.list_stride = list_stride;
  if (acc_out) {
    p.sh_m = m_out;
    p.sh_l = l_out;
    p.sh_acc = acc_out;
    return v3_common(p, q, q_dtype, q_seq_stride, q_head_stride, keys, k_dtype, k_seq_stride, k_head_stride,
                     k_tok_stride, values, v_dtype, v_seq_stride, v_head_stride, v_tok_stride, num_seqs,
                     num_kv_heads, group, seq_len, head_dim, 1, num_sms, nullptr, OC_F32, 0, head_dim, nullptr,
                     retained, status, workspace, workspace_bytes, stream);
  }
  return v3_common(p, q, q_dtype, q_seq_stride, q_head_stride, keys, k_dtype, k_seq_stride, k_head_stride,
                   k_tok_stride, values, v_dtype, v_seq_stride, v_head_stride, v_tok_stride, num_seqs,
                   num_kv_heads, group, seq_len, head_dim, 1, num_sms, out, out_dtype, out_seq_stride,
                   out_head_stride, nullptr, retained, status, workspace, workspace_bytes, stream);
}

}  // extern "C"
