// capi.cu -- extern "C" entry points of libmxfa_b200.so (see include/mxfa_b200.h).
//
// Host-side responsibilities only: argument guards with the reference's
// return codes, the split plan, TMA tensor-map encoding (through the driver
// entry point, so the library needs no libcuda link), per-device kernel
// attributes, and stream-ordered launches.  No entry point synchronises or
// reads device memory on the host except mxfa_read_error_flags.
#include <cudaTypedefs.h>

#include <atomic>
#include <climits>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include <cstdlib>

#include "decode.cuh"
#include "prefill_sm100.cuh"

namespace mxfa {

namespace {

thread_local char g_last_error[512] = {0};

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MXFA_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
  return MXFA_OK;
}

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

int sm_count() {
  static std::atomic<int> cache[64];
  const int dev = current_device();
  if (dev >= 0 && dev < 64) {
    int v = cache[dev].load(std::memory_order_relaxed);
    if (v > 0) return v;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  if (dev >= 0 && dev < 64) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

// Opt a kernel into > 48 KB dynamic shared memory once per device.
template <typename K>
int ensure_smem(K kernel, int bytes, std::atomic<unsigned long long>& done) {
  const int dev = current_device();
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return MXFA_OK;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return fail(MXFA_ERR_CUDA, "cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
  done.fetch_or(bit, std::memory_order_acq_rel);
  return MXFA_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 3-D map over a [rows][heads][D] tensor with a (64 columns, 1 head,
// box_rows rows) box and 128-byte swizzle.
bool encode_rows_map(CUtensorMap* map, const void* base, int D, int heads, long long rows, int box_rows) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
  if (rows <= 0 || rows > 0xFFFFFFFFll) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(heads) * D * 2};
  cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 3-D map over a KV cache viewed as [slots = P*PS][HKV][D] with a
// (64 columns, 1 head, 16 slots) box and 128-byte swizzle.
// 4-D view of the same cache for whole-tile boxes: dims (64 columns, head,
// slot row, 64-column block) with byte strides (D*2, HKV*D*2, 128); the box
// (64, 1, 16, D/64) lands in shared memory as [block][row][128 B], exactly
// the layout two 3-D boxes produce, in one copy instead of D/64.
// 5-D view over BOTH caches for one box per K+V tile: the 4-D view above
// plus a fifth dimension of extent 2 whose stride is the byte distance from
// the lower of the two caches to the higher.  The box lands as [K|V][block]
// [row][128 B] (V first when V lies below K, reported through *swap).  Any
// in-range coordinate addresses an element of K or V; rows past the caches
// are zero-filled without a read, as with the other maps.
bool encode_kv_map_5d(CUtensorMap* map, const void* k, const void* v, int D, int HKV, long long slots,
                      int* swap) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  const uintptr_t ka = reinterpret_cast<uintptr_t>(k), va = reinterpret_cast<uintptr_t>(v);
  if (((ka | va) & 15) != 0 || ka == va) return false;
  if (slots <= 0 || slots > 0xFFFFFFFFll) return false;
  const uintptr_t lo = ka < va ? ka : va;
  const unsigned long long dist = ka < va ? va - ka : ka - va;
  if (dist >= (1ull << 40)) return false;  // tensor-map stride limit
  cuuint64_t dims[5] = {64, static_cast<cuuint64_t>(HKV), static_cast<cuuint64_t>(slots),
                        static_cast<cuuint64_t>(D / 64), 2};
  cuuint64_t strides[4] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(HKV) * D * 2, 128,
                           static_cast<cuuint64_t>(dist)};
  cuuint32_t box[5] = {64, 1, static_cast<cuuint32_t>(kTileTok), static_cast<cuuint32_t>(D / 64), 2};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 5, reinterpret_cast<void*>(lo), dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  *swap = va < ka ? 1 : 0;
  return true;
}

bool encode_kv_map_4d(CUtensorMap* map, const void* base, int D, int HKV, long long slots) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
  if (slots <= 0 || slots > 0xFFFFFFFFll) return false;
  cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(HKV), static_cast<cuuint64_t>(slots),
                        static_cast<cuuint64_t>(D / 64)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(HKV) * D * 2, 128};
  cuuint32_t box[4] = {64, 1, static_cast<cuuint32_t>(kTileTok), static_cast<cuuint32_t>(D / 64)};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, const_cast<void*>(base), dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool encode_kv_map(CUtensorMap* map, const void* base, int D, int HKV, long long slots) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
  if (slots <= 0 || slots > 0xFFFFFFFFll) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(HKV), static_cast<cuuint64_t>(slots)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(HKV) * D * 2};
  cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(kTileTok)};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// ------------------------------------------------------------------ decode

// Whether the last decode launch on this thread merged a context-parallel
// step in place (cp_merge kept) or left the merge to cp_merge_kernel.
thread_local int g_cp_merged = 0;

template <typename T, int HD, int NT, bool kTma, bool kFp8 = false>
int launch_decode_inst(const DecodeParams& p, dim3 grid, const CUtensorMap& tk, const CUtensorMap& tv,
                       cudaStream_t st) {
  static std::atomic<unsigned long long> done{0};
  auto kern = paged_decode_kernel<T, HD, NT, kTma, kFp8>;
  const int smem = DecodeCfg<HD, NT, kFp8>::kSmemBytes;
  if (int rc = ensure_smem(kern, smem, done)) return rc;
  DecodeParams pl = p;
  if (pl.cp_merge) {
    // A unit's merging CTA waits for the other ranks while holding its SM
    // slot.  With fewer units than resident CTAs the rest of the grid always
    // has room to run, so every rank publishes every unit and every wait
    // ends; otherwise the merge goes to its own kernel.
    static std::atomic<int> per_sm{-1};
    int occ = per_sm.load(std::memory_order_relaxed);
    if (occ < 0) {
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kDecThreads, smem) != cudaSuccess) occ = 0;
      per_sm.store(occ, std::memory_order_relaxed);
    }
    if (static_cast<long long>(pl.B) * grid.x >= static_cast<long long>(occ) * sm_count()) pl.cp_merge = 0;
  }
  g_cp_merged = pl.cp_merge;
  // programmatic dependent launch (the kernel waits for its predecessor
  // before reading inputs, and releases its successor early)
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, pl, tk, tv);
  if (e != cudaSuccess) return fail(MXFA_ERR_CUDA, "paged_decode_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("paged_decode_kernel");
}

template <typename T, int HD>
int launch_decode_t(const DecodeParams& p, int nt, bool tma, dim3 grid, const CUtensorMap& tk,
                    const CUtensorMap& tv, cudaStream_t st) {
  if (nt == 1)
    return tma ? launch_decode_inst<T, HD, 1, true>(p, grid, tk, tv, st)
               : launch_decode_inst<T, HD, 1, false>(p, grid, tk, tv, st);
  return tma ? launch_decode_inst<T, HD, 2, true>(p, grid, tk, tv, st)
             : launch_decode_inst<T, HD, 2, false>(p, grid, tk, tv, st);
}

template <typename T>
int launch_decode_fp8(const DecodeParams& p, int nt, bool tma, dim3 grid, const CUtensorMap& tk,
                      const CUtensorMap& tv, cudaStream_t st) {
  if (nt == 1)
    return tma ? launch_decode_inst<T, 128, 1, true, true>(p, grid, tk, tv, st)
               : launch_decode_inst<T, 128, 1, false, true>(p, grid, tk, tv, st);
  return tma ? launch_decode_inst<T, 128, 2, true, true>(p, grid, tk, tv, st)
             : launch_decode_inst<T, 128, 2, false, true>(p, grid, tk, tv, st);
}

// 4-D view over BOTH e4m3 caches (D = 128: one 128-byte row per head): dims
// (128 bytes, head, slot row, K|V) with byte strides (128, HKV*128, distance
// between the caches); the box (128, 1, 16, 2) is a whole K+V tile.
bool encode_kv_map_fp8(CUtensorMap* map, const void* k, const void* v, int HKV, long long slots, int* swap) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  const uintptr_t ka = reinterpret_cast<uintptr_t>(k), va = reinterpret_cast<uintptr_t>(v);
  if (((ka | va) & 15) != 0 || ka == va) return false;
  if (slots <= 0 || slots > 0xFFFFFFFFll) return false;
  const uintptr_t lo = ka < va ? ka : va;
  const unsigned long long dist = ka < va ? va - ka : ka - va;
  if (dist >= (1ull << 40)) return false;
  cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(HKV), static_cast<cuuint64_t>(slots), 2};
  cuuint64_t strides[3] = {128, static_cast<cuuint64_t>(HKV) * 128, static_cast<cuuint64_t>(dist)};
  cuuint32_t box[4] = {128, 1, static_cast<cuuint32_t>(kTileTok), 2};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, reinterpret_cast<void*>(lo), dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  *swap = va < ka ? 1 : 0;
  return true;
}

// Encoded tensor maps of recently used operands, keyed by everything the
// encoding reads (device, addresses, shape, element type), so a call reuses
// them instead of re-encoding (one driver call per map).  Hash tables per
// kind, bounded: when one reaches its limit it is cleared and refilled, so a
// model with many layers' caches still hits on every call after the first.
struct MapKey {
  int device;
  const void *a, *b, *c;
  long long n0, n1, n2, n3;
  bool operator==(const MapKey& o) const {
    return device == o.device && a == o.a && b == o.b && c == o.c && n0 == o.n0 && n1 == o.n1 && n2 == o.n2 &&
           n3 == o.n3;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<int>()(k.device);
    auto mix = [&h](size_t v) { h ^= v + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2); };
    mix(std::hash<const void*>()(k.a));
    mix(std::hash<const void*>()(k.b));
    mix(std::hash<const void*>()(k.c));
    mix(std::hash<long long>()(k.n0));
    mix(std::hash<long long>()(k.n1));
    mix(std::hash<long long>()(k.n2));
    mix(std::hash<long long>()(k.n3));
    return h;
  }
};
template <typename V>
struct MapCache {
  std::mutex mu;
  std::unordered_map<MapKey, V, MapKeyHash> table;
  size_t limit;
  explicit MapCache(size_t lim) : limit(lim) {}
  bool get(const MapKey& k, V* out) {
    std::lock_guard<std::mutex> lock(mu);
    auto it = table.find(k);
    if (it == table.end()) return false;
    *out = it->second;
    return true;
  }
  void put(const MapKey& k, const V& v) {
    std::lock_guard<std::mutex> lock(mu);
    if (table.size() >= limit) table.clear();
    table[k] = v;
  }
};

struct KvMaps {
  CUtensorMap tk{}, tv{};
  int kind = 0, swap = 0;
  bool tma = false;
};
MapCache<KvMaps> g_kv_maps(8192);

bool kv_map_cache_get(const void* k, const void* v, int D, int HKV, long long slots, bool fp8, KvMaps* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  return g_kv_maps.get(MapKey{dev, k, v, nullptr, D, HKV, slots, fp8 ? 1 : 0}, out);
}

void kv_map_cache_put(const void* k, const void* v, int D, int HKV, long long slots, bool fp8, const KvMaps& maps) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return;
  g_kv_maps.put(MapKey{dev, k, v, nullptr, D, HKV, slots, fp8 ? 1 : 0}, maps);
}

// The three maps of a prefill call (q, k, v rows).
struct PrefillMaps {
  CUtensorMap q{}, k{}, v{};
};
MapCache<PrefillMaps> g_prefill_maps(4096);

// Runs the decode kernel (split or direct) for a validated configuration;
// kv_fp8: the caches hold e4m3 (D = 128 only).
int run_decode(DecodeParams p, int D, bool bf16, cudaStream_t st, bool kv_fp8 = false) {
  const int rows_kv = p.Sq * p.GQ;
  const int nt = rows_kv <= 8 ? 1 : 2;
  const int row_groups = (rows_kv + 8 * nt - 1) / (8 * nt);
  const int nz = p.ows != nullptr ? p.NP : 1;
  if (nz > 65535 || p.B > 65535) return fail(MXFA_ERR_UNSUPPORTED, "too many splits or sequences");
  dim3 grid(p.HKV * row_groups, p.B, nz);
  CUtensorMap tk, tv;
  std::memset(&tk, 0, sizeof(tk));
  std::memset(&tv, 0, sizeof(tv));
  bool tma = (p.PS % kTileTok) == 0;
  const long long slots = static_cast<long long>(p.P) * p.PS;
  KvMaps maps;
  if (tma && !kv_map_cache_get(p.k, p.v, D, p.HKV, slots, kv_fp8, &maps)) {
    maps = KvMaps{};
    if (kv_fp8) {
      maps.tma = D == 128 && encode_kv_map_fp8(&maps.tk, p.k, p.v, p.HKV, slots, &maps.swap);
    } else if (encode_kv_map_5d(&maps.tk, p.k, p.v, D, p.HKV, slots, &maps.swap)) {
      // fewest copies per tile that the driver accepts: K+V in one box, else
      // one box per cache, else one per 64-column block
      maps.kind = 5;
      maps.tma = true;
    } else if (encode_kv_map_4d(&maps.tk, p.k, D, p.HKV, slots) && encode_kv_map_4d(&maps.tv, p.v, D, p.HKV, slots)) {
      maps.kind = 4;
      maps.tma = true;
    } else {
      maps.kind = 3;
      maps.tma = encode_kv_map(&maps.tk, p.k, D, p.HKV, slots) && encode_kv_map(&maps.tv, p.v, D, p.HKV, slots);
    }
    kv_map_cache_put(p.k, p.v, D, p.HKV, slots, kv_fp8, maps);
  }
  if (tma) {
    tma = maps.tma;
    tk = maps.tk;
    tv = maps.tv;
    p.kv_map = maps.kind;
    p.kv_swap = maps.swap;
  }
  if (kv_fp8) {
    if (D != 128) return fail(MXFA_ERR_UNSUPPORTED, "FP8 caches need head dim 128 (got %d)", D);
    if (!tma) p.kv_swap = 0;
    return bf16 ? launch_decode_fp8<__nv_bfloat16>(p, nt, tma, grid, tk, tv, st)
                : launch_decode_fp8<__half>(p, nt, tma, grid, tk, tv, st);
  }
  if (bf16)
    return D == 128 ? launch_decode_t<__nv_bfloat16, 128>(p, nt, tma, grid, tk, tv, st)
                    : launch_decode_t<__nv_bfloat16, 64>(p, nt, tma, grid, tk, tv, st);
  return D == 128 ? launch_decode_t<__half, 128>(p, nt, tma, grid, tk, tv, st)
                  : launch_decode_t<__half, 64>(p, nt, tma, grid, tk, tv, st);
}

template <typename T, int HD, bool kPacked>
int launch_combine_inst(const float* ows, const float* mdws, void* out, float* out_f32, float* lse, int rows,
                        int NP, cudaStream_t st) {
  split_combine_kernel<T, HD, kPacked>
      <<<(rows + 3) / 4, 128, 0, st>>>(ows, mdws, static_cast<T*>(out), out_f32, lse, rows, NP);
  return check_launch("split_combine_kernel");
}

template <bool kPacked>
int run_combine(const float* ows, const float* mdws, void* out, float* out_f32, float* lse, int rows, int D,
                int NP, bool bf16, cudaStream_t st) {
  if (rows == 0) return MXFA_OK;
  if (bf16)
    return D == 128 ? launch_combine_inst<__nv_bfloat16, 128, kPacked>(ows, mdws, out, out_f32, lse, rows, NP, st)
                    : launch_combine_inst<__nv_bfloat16, 64, kPacked>(ows, mdws, out, out_f32, lse, rows, NP, st);
  return D == 128 ? launch_combine_inst<__half, 128, kPacked>(ows, mdws, out, out_f32, lse, rows, NP, st)
                  : launch_combine_inst<__half, 64, kPacked>(ows, mdws, out, out_f32, lse, rows, NP, st);
}

// Split plan: enough CTAs to fill every SM twice, chunks of >= 256 positions.
void plan_splits(int B, int HKV, int row_groups, int max_len, int* np_out, int* clen_out) {
  const long long units = static_cast<long long>(B) * HKV * row_groups;
  const long long target = 2LL * sm_count();
  int np = 1;
  if (units > 0 && units < target && max_len > 256) {
    np = static_cast<int>((target + units - 1) / units);
    const int cap = (max_len + 255) / 256;
    if (np > cap) np = cap;
    if (np > 1024) np = 1024;
  }
  if (np < 1) np = 1;
  int clen = (max_len + np - 1) / np;
  clen = ((clen + kTileTok - 1) / kTileTok) * kTileTok;
  if (clen < kTileTok) clen = kTileTok;
  np = (max_len + clen - 1) / clen;
  if (np < 1) np = 1;
  *np_out = np;
  *clen_out = clen;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3) == 0; }

// Positions a sequence can hold (block-table width x page size, or one page
// without a table); positions are 32-bit indices in the kernels.
int cache_capacity(const void* block_table, int BTW, int PS, int* cap) {
  const long long c = block_table ? static_cast<long long>(BTW) * PS : PS;
  if (c > INT_MAX) return fail(MXFA_ERR_UNSUPPORTED, "cache capacity %lld positions above 2^31-1", c);
  *cap = static_cast<int>(c);
  return MXFA_OK;
}

template <int HD>
int launch_packed_combine(const float* ows, const float* mdws, float* packed, int rows, int NP, cudaStream_t st) {
  if (rows == 0) return MXFA_OK;
  split_combine_kernel<__nv_bfloat16, HD, false, true>
      <<<(rows + 3) / 4, 128, 0, st>>>(ows, mdws, nullptr, packed, nullptr, rows, NP);
  return check_launch("split_combine_kernel(packed)");
}

}  // namespace
}  // namespace mxfa

using namespace mxfa;

extern "C" {

int mxfa_abi_version(void) { return 1; }

const char* mxfa_last_error(void) { return g_last_error; }

int mxfa_is_available(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  cudaGetLastError();
  return (major == 10 && minor == 0) ? 1 : 0;
}

int mxfa_read_error_flags(unsigned int* flags) {
  if (flags == nullptr) return fail(MXFA_ERR_INVALID, "flags is NULL");
  unsigned int v = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_error_flags, sizeof(v));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_error_flags, &zero, sizeof(zero));
  if (e != cudaSuccess) return fail(MXFA_ERR_CUDA, "reading error flags failed: %s", cudaGetErrorString(e));
  *flags = v;
  return MXFA_OK;
}

size_t mxfa_split_workspace_bytes(int rows, int D, int NP) {
  if (rows <= 0 || D <= 0 || NP <= 0) return 0;
  return static_cast<size_t>(rows) * NP * (static_cast<size_t>(D) + 2) * sizeof(float);
}

int mxfa_kvcache_plan(int B, int Sq, int HQ, int HKV, int D, int max_len, int* num_splits, int* chunk_len) {
  if (num_splits == nullptr || chunk_len == nullptr) return fail(MXFA_ERR_INVALID, "null output pointer");
  if (B <= 0 || Sq <= 0 || HQ <= 0 || HKV <= 0 || HQ % HKV != 0 || max_len < 0)
    return fail(MXFA_ERR_INVALID, "invalid plan arguments");
  (void)D;
  const int rows_kv = Sq * (HQ / HKV);
  const int nt = rows_kv <= 8 ? 1 : 2;
  const int row_groups = (rows_kv + 8 * nt - 1) / (8 * nt);
  plan_splits(B, HKV, row_groups, max_len < 1 ? 1 : max_len, num_splits, chunk_len);
  return MXFA_OK;
}

static int kvcache_attention_impl(const void* q, const void* k_cache, const void* v_cache,
                                  const int32_t* block_table, const int32_t* seqlens, void* out, float* lse,
                                  void* workspace, size_t workspace_bytes, int B, int Sq, int HQ, int HKV, int D,
                                  int PS, int BTW, int num_pages, int append_len, int num_splits, int chunk_len,
                                  int causal, int bf16, float scale, const void* k_new, const void* v_new,
                                  unsigned* counters, void* stream, bool kv_fp8 = false, float k_scale = 1.f,
                                  float v_scale = 1.f, const int32_t* order = nullptr) {
  if (D != 64 && D != 128) return fail(MXFA_ERR_UNSUPPORTED, "head dim %d not in {64, 128}", D);
  if (B < 0 || Sq < 0 || HQ <= 0 || HKV <= 0 || HQ % HKV != 0)
    return fail(MXFA_ERR_INVALID, "bad head / batch geometry (B=%d Sq=%d HQ=%d HKV=%d)", B, Sq, HQ, HKV);
  if (B == 0 || Sq == 0) return MXFA_OK;
  if (PS <= 0 || num_pages <= 0 || append_len < 0) return fail(MXFA_ERR_INVALID, "bad cache geometry");
  if (block_table != nullptr && BTW <= 0) return fail(MXFA_ERR_INVALID, "block table width must be positive");
  if (!q || !k_cache || !v_cache || !seqlens || !out) return fail(MXFA_ERR_INVALID, "null tensor pointer");
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || (reinterpret_cast<uintptr_t>(out) & 7))
    return fail(MXFA_ERR_INVALID, "tensors must be 16-byte aligned (out 8-byte)");
  const long long rows = static_cast<long long>(B) * Sq * HQ;
  if (rows > INT_MAX) return fail(MXFA_ERR_UNSUPPORTED, "%lld query rows (B*Sq*HQ) above 2^31-1", rows);
  DecodeParams p{};
  p.q = q;
  p.k = k_cache;
  p.v = v_cache;
  p.bt = block_table;
  p.seqlens = seqlens;
  p.out = out;
  p.lse = lse;
  p.B = B;
  p.Sq = Sq;
  p.HQ = HQ;
  p.HKV = HKV;
  p.PS = PS;
  p.BTW = block_table ? BTW : 1;
  p.P = num_pages;
  p.GQ = HQ / HKV;
  p.append_len = append_len;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * kLog2e * (kv_fp8 ? k_scale : 1.f);
  p.v_scale = kv_fp8 ? v_scale : 1.f;
  p.k_new = k_new;
  p.v_new = v_new;
  p.order = order;
  int max_len = 0;
  if (int rc = cache_capacity(block_table, BTW, PS, &max_len)) return rc;
  if (num_splits <= 0 || chunk_len <= 0) {
    mxfa_kvcache_plan(B, Sq, HQ, HKV, D, max_len, &num_splits, &chunk_len);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (num_splits <= 1) {
    p.NP = 1;
    p.c_len = max_len;
    return run_decode(p, D, bf16 != 0, st, kv_fp8);
  }
  const size_t need = mxfa_split_workspace_bytes(static_cast<int>(rows), D, num_splits);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
    return fail(MXFA_ERR_INVALID, "split workspace too small or unaligned (%zu < %zu bytes)", workspace_bytes, need);
  if (static_cast<long long>(num_splits) * chunk_len < max_len)
    return fail(MXFA_ERR_INVALID, "%d splits of %d positions do not cover the cache capacity %d", num_splits,
                chunk_len, max_len);
  p.NP = num_splits;
  p.c_len = chunk_len;
  p.ows = static_cast<float*>(workspace);
  p.mdws = p.ows + rows * num_splits * D;
  if (counters != nullptr) {
    // one launch: the last split CTA of every unit merges the partials
    if (reinterpret_cast<uintptr_t>(counters) & 3) return fail(MXFA_ERR_INVALID, "counters must be 4-byte aligned");
    p.counters = counters;
    return run_decode(p, D, bf16 != 0, st, kv_fp8);
  }
  if (int rc = run_decode(p, D, bf16 != 0, st, kv_fp8)) return rc;
  return run_combine<false>(p.ows, p.mdws, out, nullptr, lse, static_cast<int>(rows), D, num_splits, bf16 != 0, st);
}

size_t mxfa_split_counter_bytes(int B, int Sq, int HQ, int HKV) {
  if (B <= 0 || Sq <= 0 || HKV <= 0 || HQ <= 0 || HQ % HKV != 0) return 0;
  const int rows_kv = Sq * (HQ / HKV);
  const int nt = rows_kv <= 8 ? 1 : 2;
  const long long groups = (rows_kv + 8 * nt - 1) / (8 * nt);
  return static_cast<size_t>(B) * HKV * groups * sizeof(unsigned);
}

int mxfa_kvcache_attention_counted_launch(const void* q, const void* k_cache, const void* v_cache,
                                          const int32_t* block_table, const int32_t* seqlens, void* out, float* lse,
                                          void* workspace, size_t workspace_bytes, unsigned* counters, int B, int Sq,
                                          int HQ, int HKV, int D, int PS, int BTW, int num_pages, int append_len,
                                          int num_splits, int chunk_len, int causal, int bf16, float scale,
                                          void* stream) {
  if (counters == nullptr) return fail(MXFA_ERR_INVALID, "counters is NULL");
  return kvcache_attention_impl(q, k_cache, v_cache, block_table, seqlens, out, lse, workspace, workspace_bytes, B,
                                Sq, HQ, HKV, D, PS, BTW, num_pages, append_len, num_splits, chunk_len, causal, bf16,
                                scale, nullptr, nullptr, counters, stream);
}

int mxfa_kvcache_attention_launch(const void* q, const void* k_cache, const void* v_cache,
                                  const int32_t* block_table, const int32_t* seqlens, void* out, float* lse,
                                  void* workspace, size_t workspace_bytes, int B, int Sq, int HQ, int HKV, int D,
                                  int PS, int BTW, int num_pages, int append_len, int num_splits, int chunk_len,
                                  int causal, int bf16, float scale, void* stream) {
  return kvcache_attention_impl(q, k_cache, v_cache, block_table, seqlens, out, lse, workspace, workspace_bytes, B,
                                Sq, HQ, HKV, D, PS, BTW, num_pages, append_len, num_splits, chunk_len, causal, bf16,
                                scale, nullptr, nullptr, nullptr, stream);
}

int mxfa_kvcache_attention_fp8_launch(const void* q, const void* k_cache, const void* v_cache,
                                      const int32_t* block_table, const int32_t* seqlens, void* out, float* lse,
                                      void* workspace, size_t workspace_bytes, unsigned* counters, int B, int Sq,
                                      int HQ, int HKV, int D, int PS, int BTW, int num_pages, int append_len,
                                      int num_splits, int chunk_len, int causal, int bf16, float scale,
                                      float k_scale, float v_scale, void* stream) {
  if (!(k_scale > 0.f) || !(v_scale > 0.f) || !std::isfinite(k_scale) || !std::isfinite(v_scale))
    return fail(MXFA_ERR_INVALID, "k_scale / v_scale must be positive and finite");
  return kvcache_attention_impl(q, k_cache, v_cache, block_table, seqlens, out, lse, workspace, workspace_bytes, B,
                                Sq, HQ, HKV, D, PS, BTW, num_pages, append_len, num_splits, chunk_len, causal, bf16,
                                scale, nullptr, nullptr, counters, stream, true, k_scale, v_scale);
}

int mxfa_kvcache_append_attention_launch(const void* q, void* k_cache, void* v_cache,
                                         const int32_t* block_table, const int32_t* seqlens, void* out, float* lse,
                                         void* workspace, size_t workspace_bytes, unsigned* counters,
                                         const void* k_new, const void* v_new, int B, int Sq, int HQ, int HKV, int D, int PS, int BTW,
                                         int num_pages, int append_len, int num_splits, int chunk_len, int causal,
                                         int bf16, float scale, void* stream) {
  if (k_new == nullptr || v_new == nullptr || append_len <= 0)
    return fail(MXFA_ERR_INVALID, "fused append needs k_new, v_new and append_len > 0");
  if (HKV <= 0 || HQ % HKV != 0 || Sq * (HQ / HKV) > 16)
    return fail(MXFA_ERR_UNSUPPORTED, "fused append covers up to 16 query rows per KV head (Sq*GQ=%d)",
                HKV > 0 ? Sq * (HQ / HKV) : 0);
  if (!aligned16(k_new) || !aligned16(v_new) || (D * 2) % 16 != 0)
    return fail(MXFA_ERR_INVALID, "appended rows must be 16-byte aligned");
  return kvcache_attention_impl(q, k_cache, v_cache, block_table, seqlens, out, lse, workspace, workspace_bytes,
                                B, Sq, HQ, HKV, D, PS, BTW, num_pages, append_len, num_splits, chunk_len, causal,
                                bf16, scale, k_new, v_new, counters, stream);
}

int mxfa_kvcache_length_order_launch(const int32_t* seqlens, int B, int32_t* order, void* stream) {
  if (B <= 0) return MXFA_OK;
  if (B > kRankMaxBatch) return fail(MXFA_ERR_UNSUPPORTED, "length order covers up to %d sequences", kRankMaxBatch);
  if (seqlens == nullptr || order == nullptr) return fail(MXFA_ERR_INVALID, "null pointer");
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kRankMaxBatch);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, length_order_kernel, seqlens, B, order);
  if (e != cudaSuccess) return fail(MXFA_ERR_CUDA, "length_order_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("length_order_kernel");
}

int mxfa_kvcache_attention_ordered_launch(const void* q, const void* k_cache, const void* v_cache,
                                          const int32_t* block_table, const int32_t* seqlens,
                                          const int32_t* length_order, void* out, float* lse, void* workspace,
                                          size_t workspace_bytes, unsigned* counters, int B, int Sq, int HQ, int HKV,
                                          int D, int PS, int BTW, int num_pages, int append_len, int num_splits,
                                          int chunk_len, int causal, int bf16, float scale, int kv_fp8,
                                          float k_scale, float v_scale, void* stream) {
  if (kv_fp8 && (!(k_scale > 0.f) || !(v_scale > 0.f) || !std::isfinite(k_scale) || !std::isfinite(v_scale)))
    return fail(MXFA_ERR_INVALID, "k_scale / v_scale must be positive and finite");
  return kvcache_attention_impl(q, k_cache, v_cache, block_table, seqlens, out, lse, workspace, workspace_bytes, B,
                                Sq, HQ, HKV, D, PS, BTW, num_pages, append_len, num_splits, chunk_len, causal, bf16,
                                scale, nullptr, nullptr, counters, stream, kv_fp8 != 0, k_scale, v_scale,
                                length_order);
}

// ------------------------------------------------ context-parallel exchange

size_t mxfa_cp_buffer_bytes(int world, int B, int HQ, int HKV, int D) {
  if (world <= 0 || B <= 0 || HKV <= 0 || HQ <= 0 || HQ % HKV != 0 || (D != 64 && D != 128)) return 0;
  if (static_cast<long long>(B) * HQ > INT_MAX) return 0;
  return cp_layout(world, B * HQ, D).bytes;
}

int mxfa_peer_alloc(size_t bytes, void** ptr) {
  if (ptr == nullptr || bytes == 0) return fail(MXFA_ERR_INVALID, "bad peer allocation request");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return fail(MXFA_ERR_CUDA, "peer buffer allocation: %s", cudaGetErrorString(e));
  }
  *ptr = p;
  return MXFA_OK;
}

int mxfa_peer_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? MXFA_OK : fail(MXFA_ERR_CUDA, "peer buffer free: %s", cudaGetErrorString(e));
}

int mxfa_peer_export(void* ptr, void* handle) {
  if (ptr == nullptr || handle == nullptr) return fail(MXFA_ERR_INVALID, "null pointer");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return fail(MXFA_ERR_CUDA, "IPC export: %s", cudaGetErrorString(e));
  std::memcpy(handle, &h, sizeof(h));
  return MXFA_OK;
}

int mxfa_peer_import(const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return fail(MXFA_ERR_INVALID, "null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(MXFA_ERR_CUDA, "IPC import: %s", cudaGetErrorString(e));
  *ptr = p;
  return MXFA_OK;
}

int mxfa_peer_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? MXFA_OK : fail(MXFA_ERR_CUDA, "IPC close: %s", cudaGetErrorString(e));
}

static int cp_decode_impl(const void* q, const void* k_cache, const void* v_cache, const int32_t* block_table,
                          const int32_t* seqlens, void* out, float* lse, void* workspace, size_t workspace_bytes,
                          unsigned* counters, const unsigned long long* peer_bufs, int rank, int world, int B,
                          int HQ, int HKV, int D, int PS, int BTW, int num_pages, int num_splits, int chunk_len,
                          int bf16, float scale, void* stream, void* local_buf) {
  if (peer_bufs == nullptr || counters == nullptr) return fail(MXFA_ERR_INVALID, "peer buffers / counters missing");
  if (world < 1 || world > 32 || rank < 0 || rank >= world)
    return fail(MXFA_ERR_INVALID, "rank %d of world %d (1..32 ranks)", rank, world);
  if (HKV <= 0 || HQ % HKV != 0 || HQ / HKV > 16)
    return fail(MXFA_ERR_UNSUPPORTED, "context-parallel decode covers up to 16 query heads per KV head");
  if (D != 64 && D != 128) return fail(MXFA_ERR_UNSUPPORTED, "head dim %d not in {64, 128}", D);
  if (B <= 0) return MXFA_OK;
  if (PS <= 0 || num_pages <= 0) return fail(MXFA_ERR_INVALID, "bad cache geometry");
  if (block_table != nullptr && BTW <= 0) return fail(MXFA_ERR_INVALID, "block table width must be positive");
  if (!q || !k_cache || !v_cache || !seqlens || !out) return fail(MXFA_ERR_INVALID, "null tensor pointer");
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || (reinterpret_cast<uintptr_t>(out) & 7) ||
      !aligned16(local_buf))
    return fail(MXFA_ERR_INVALID, "tensors and the exchange buffer must be 16-byte aligned (out 8-byte)");
  const long long rows = static_cast<long long>(B) * HQ;
  if (rows > INT_MAX) return fail(MXFA_ERR_UNSUPPORTED, "%lld query rows (B*HQ) above 2^31-1", rows);
  int max_len = 0;
  if (int rc = cache_capacity(block_table, BTW, PS, &max_len)) return rc;
  if (num_splits <= 0 || chunk_len <= 0) mxfa_kvcache_plan(B, 1, HQ, HKV, D, max_len, &num_splits, &chunk_len);
  const size_t need = mxfa_split_workspace_bytes(static_cast<int>(rows), D, num_splits);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
    return fail(MXFA_ERR_INVALID, "split workspace too small or unaligned (%zu < %zu bytes)", workspace_bytes, need);
  if (static_cast<long long>(num_splits) * chunk_len < max_len)
    return fail(MXFA_ERR_INVALID, "%d splits of %d positions do not cover the cache capacity %d", num_splits,
                chunk_len, max_len);
  DecodeParams p{};
  p.q = q;
  p.k = k_cache;
  p.v = v_cache;
  p.bt = block_table;
  p.seqlens = seqlens;
  p.out = out;
  p.lse = lse;
  p.B = B;
  p.Sq = 1;
  p.HQ = HQ;
  p.HKV = HKV;
  p.PS = PS;
  p.BTW = block_table ? BTW : 1;
  p.P = num_pages;
  p.GQ = HQ / HKV;
  p.causal = 0;
  p.scale_log2 = scale * kLog2e;
  p.v_scale = 1.f;
  p.NP = num_splits;
  p.c_len = chunk_len;
  p.ows = static_cast<float*>(workspace);
  p.mdws = p.ows + rows * num_splits * D;
  p.counters = counters;
  p.cp_bufs = peer_bufs;
  p.cp_rank = rank;
  p.cp_world = world;
  p.cp_merge = local_buf != nullptr ? 1 : 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  g_cp_merged = 0;
  if (int rc = run_decode(p, D, bf16 != 0, st)) return rc;
  if (local_buf == nullptr || g_cp_merged) return MXFA_OK;
  return mxfa_cp_merge_launch(local_buf, out, lse, world, B, HQ, HKV, D, bf16, stream);
}

int mxfa_cp_decode_launch(const void* q, const void* k_cache, const void* v_cache, const int32_t* block_table,
                          const int32_t* seqlens, void* out, float* lse, void* workspace, size_t workspace_bytes,
                          unsigned* counters, const unsigned long long* peer_bufs, int rank, int world, int B,
                          int HQ, int HKV, int D, int PS, int BTW, int num_pages, int num_splits, int chunk_len,
                          int bf16, float scale, void* stream) {
  return cp_decode_impl(q, k_cache, v_cache, block_table, seqlens, out, lse, workspace, workspace_bytes, counters,
                        peer_bufs, rank, world, B, HQ, HKV, D, PS, BTW, num_pages, num_splits, chunk_len, bf16, scale,
                        stream, nullptr);
}

int mxfa_cp_last_merged_in_place(void) { return g_cp_merged; }

int mxfa_cp_attention_launch(const void* q, const void* k_cache, const void* v_cache, const int32_t* block_table,
                             const int32_t* seqlens, void* out, float* lse, void* workspace, size_t workspace_bytes,
                             unsigned* counters, const unsigned long long* peer_bufs, void* local_buf, int rank,
                             int world, int B, int HQ, int HKV, int D, int PS, int BTW, int num_pages, int num_splits,
                             int chunk_len, int bf16, float scale, void* stream) {
  if (local_buf == nullptr) return fail(MXFA_ERR_INVALID, "local exchange buffer missing");
  return cp_decode_impl(q, k_cache, v_cache, block_table, seqlens, out, lse, workspace, workspace_bytes, counters,
                        peer_bufs, rank, world, B, HQ, HKV, D, PS, BTW, num_pages, num_splits, chunk_len, bf16, scale,
                        stream, local_buf);
}

int mxfa_cp_merge_launch(void* local_buf, void* out, float* lse, int world, int B, int HQ, int HKV, int D, int bf16,
                         void* stream) {
  if (local_buf == nullptr || out == nullptr) return fail(MXFA_ERR_INVALID, "null pointer");
  // the merge checks one rank's flag per lane of a warp: at most 32 ranks,
  // as mxfa_cp_decode_launch
  if (world < 1 || world > 32) return fail(MXFA_ERR_INVALID, "world %d outside 1..32 ranks", world);
  if (HKV <= 0 || HQ % HKV != 0 || (D != 64 && D != 128)) return fail(MXFA_ERR_INVALID, "bad geometry");
  if (B <= 0) return MXFA_OK;
  if (static_cast<long long>(B) * HQ > INT_MAX)
    return fail(MXFA_ERR_UNSUPPORTED, "%lld query rows (B*HQ) above 2^31-1", static_cast<long long>(B) * HQ);
  const int rows = B * HQ;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((rows + 3) / 4);
  cfg.blockDim = dim3(128);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto* buf = static_cast<unsigned char*>(local_buf);
  cudaError_t e;
  if (bf16)
    e = D == 128 ? cudaLaunchKernelEx(&cfg, cp_merge_kernel<__nv_bfloat16, 128>, buf,
                                      static_cast<__nv_bfloat16*>(out), lse, rows, world)
                 : cudaLaunchKernelEx(&cfg, cp_merge_kernel<__nv_bfloat16, 64>, buf,
                                      static_cast<__nv_bfloat16*>(out), lse, rows, world);
  else
    e = D == 128 ? cudaLaunchKernelEx(&cfg, cp_merge_kernel<__half, 128>, buf, static_cast<__half*>(out), lse, rows,
                                      world)
                 : cudaLaunchKernelEx(&cfg, cp_merge_kernel<__half, 64>, buf, static_cast<__half*>(out), lse, rows,
                                      world);
  if (e != cudaSuccess) return fail(MXFA_ERR_CUDA, "cp_merge_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("cp_merge_kernel");
}

int mxfa_paged_decode_split_launch(const void* q, const void* k, const void* v, const void* bt, const void* sl,
                                   void* out, void* ows, void* mdws, float scale, int B, int HQ, int HKV, int D,
                                   int PS, int BTW, int bf16, int NP, int c_len, int um, void* stream) {
  // guards of m1_kernel.cpp:1212-1215
  if (HKV <= 0 || HQ % HKV != 0) return fail(MXFA_ERR_UNSUPPORTED, "HQ %% HKV != 0");
  if (D != 128 && D != 64) return fail(MXFA_ERR_UNSUPPORTED, "split kernel unsupported config: D=%d", D);
  const int GQ = HQ / HKV;
  if ((GQ != 2 && GQ != 4 && GQ != 8) || NP < 1)
    return fail(MXFA_ERR_UNSUPPORTED, "split kernel unsupported config: D=%d GQ=%d NP=%d", D, GQ, NP);
  (void)um;  // every softmax variant is served by the same online softmax
  if (B <= 0) return MXFA_OK;
  if (!q || !k || !v || !bt || !sl || !out || !ows || !mdws || PS <= 0 || BTW <= 0 || c_len <= 0)
    return fail(MXFA_ERR_INVALID, "invalid split-decode argument");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(ows) || (reinterpret_cast<uintptr_t>(mdws) & 7))
    return fail(MXFA_ERR_INVALID, "tensors must be 16-byte aligned");
  DecodeParams p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.bt = static_cast<const int*>(bt);
  p.seqlens = static_cast<const int*>(sl);
  p.out = out;
  p.ows = static_cast<float*>(ows);
  p.mdws = static_cast<float*>(mdws);
  p.B = B;
  p.Sq = 1;
  p.HQ = HQ;
  p.HKV = HKV;
  p.PS = PS;
  p.BTW = BTW;
  // the reference ABI carries no page count: bound the addressable slots only
  p.P = static_cast<int>(0x7FFFFFFFll / PS);
  p.GQ = GQ;
  p.NP = NP;
  p.c_len = c_len;
  p.scale_log2 = scale * kLog2e;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = run_decode(p, D, bf16 != 0, st)) return rc;
  return run_combine<false>(p.ows, p.mdws, out, nullptr, nullptr, B * HQ, D, NP, bf16 != 0, st);
}

int mxfa_kvcache_attention_packed_launch(const void* q, const void* k_cache, const void* v_cache,
                                         const int32_t* block_table, const int32_t* seqlens, float* packed,
                                         void* workspace, size_t workspace_bytes, int B, int HQ, int HKV, int D,
                                         int PS, int BTW, int num_pages, int num_splits, int chunk_len, int bf16,
                                         float scale, void* stream) {
  if (D != 64 && D != 128) return fail(MXFA_ERR_UNSUPPORTED, "head dim %d not in {64, 128}", D);
  if (B < 0 || HQ <= 0 || HKV <= 0 || HQ % HKV != 0)
    return fail(MXFA_ERR_INVALID, "bad head / batch geometry (B=%d HQ=%d HKV=%d)", B, HQ, HKV);
  if (B == 0) return MXFA_OK;
  if (PS <= 0 || num_pages <= 0) return fail(MXFA_ERR_INVALID, "bad cache geometry");
  if (block_table != nullptr && BTW <= 0) return fail(MXFA_ERR_INVALID, "block table width must be positive");
  if (!q || !k_cache || !v_cache || !seqlens || !packed) return fail(MXFA_ERR_INVALID, "null tensor pointer");
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache))
    return fail(MXFA_ERR_INVALID, "tensors must be 16-byte aligned");
  int max_len = 0;
  if (int rc = cache_capacity(block_table, BTW, PS, &max_len)) return rc;
  if (num_splits <= 0 || chunk_len <= 0) mxfa_kvcache_plan(B, 1, HQ, HKV, D, max_len, &num_splits, &chunk_len);
  if (static_cast<long long>(num_splits) * chunk_len < max_len)
    return fail(MXFA_ERR_INVALID, "%d splits of %d positions do not cover the cache capacity %d", num_splits,
                chunk_len, max_len);
  const int rows = B * HQ;
  const size_t need = mxfa_split_workspace_bytes(rows, D, num_splits);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
    return fail(MXFA_ERR_INVALID, "split workspace too small or unaligned (%zu < %zu bytes)", workspace_bytes, need);
  DecodeParams p{};
  p.q = q;
  p.k = k_cache;
  p.v = v_cache;
  p.bt = block_table;
  p.seqlens = seqlens;
  p.B = B;
  p.Sq = 1;
  p.HQ = HQ;
  p.HKV = HKV;
  p.PS = PS;
  p.BTW = block_table ? BTW : 1;
  p.P = num_pages;
  p.GQ = HQ / HKV;
  p.NP = num_splits;
  p.c_len = chunk_len;
  p.scale_log2 = scale * kLog2e;
  p.ows = static_cast<float*>(workspace);
  p.mdws = p.ows + static_cast<size_t>(rows) * num_splits * D;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = run_decode(p, D, bf16 != 0, st)) return rc;
  return D == 128 ? launch_packed_combine<128>(p.ows, p.mdws, packed, rows, num_splits, st)
                  : launch_packed_combine<64>(p.ows, p.mdws, packed, rows, num_splits, st);
}

int mxfa_split_combine_launch(const float* ows, const float* mdws, void* out, float* out_f32, float* lse, int rows,
                              int D, int NP, int bf16, void* stream) {
  if (D != 64 && D != 128) return fail(MXFA_ERR_UNSUPPORTED, "head dim %d not in {64, 128}", D);
  if (rows < 0 || NP < 1 || !ows || !mdws) return fail(MXFA_ERR_INVALID, "invalid combine argument");
  if (!aligned16(ows)) return fail(MXFA_ERR_INVALID, "ows must be 16-byte aligned");
  // output pairs are written as 4-byte words, (m, d) pairs read as floats
  if (!aligned4(mdws) || !aligned4(out) || !aligned4(out_f32) || !aligned4(lse))
    return fail(MXFA_ERR_INVALID, "mdws, out, out_f32 and lse must be 4-byte aligned");
  return run_combine<false>(ows, mdws, out, out_f32, lse, rows, D, NP, bf16 != 0,
                            static_cast<cudaStream_t>(stream));
}

int mxfa_lse_merge_launch(const float* packed, void* out, float* lse, int N, int rows, int D, int bf16,
                          void* stream) {
  if (D != 64 && D != 128) return fail(MXFA_ERR_UNSUPPORTED, "head dim %d not in {64, 128}", D);
  if (rows < 0 || N < 1 || !packed || !out) return fail(MXFA_ERR_INVALID, "invalid merge argument");
  if (!aligned4(packed) || !aligned4(out) || !aligned4(lse))
    return fail(MXFA_ERR_INVALID, "packed, out and lse must be 4-byte aligned");
  return run_combine<true>(packed, nullptr, out, nullptr, lse, rows, D, N, bf16 != 0,
                           static_cast<cudaStream_t>(stream));
}

int mxfa_kv_append_launch(const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                          const int32_t* block_table, const int32_t* seqlens, int B, int Sk, int HKV, int D, int PS,
                          int BTW, int num_pages, int elem_bytes, void* stream) {
  if (B < 0 || Sk < 0 || HKV <= 0 || D <= 0 || PS <= 0 || num_pages <= 0 || elem_bytes <= 0)
    return fail(MXFA_ERR_INVALID, "invalid append geometry");
  if (B == 0 || Sk == 0) return MXFA_OK;
  if (!k_new || !v_new || !k_cache || !v_cache || !seqlens) return fail(MXFA_ERR_INVALID, "null tensor pointer");
  const int row_bytes = D * elem_bytes;
  if (row_bytes % 16 != 0 || !aligned16(k_new) || !aligned16(v_new) || !aligned16(k_cache) || !aligned16(v_cache))
    return fail(MXFA_ERR_INVALID, "append rows must be 16-byte multiples on 16-byte aligned tensors");
  if (block_table != nullptr && BTW <= 0) return fail(MXFA_ERR_INVALID, "block table width must be positive");
  AppendParams p{};
  p.k_new = static_cast<const uint8_t*>(k_new);
  p.v_new = static_cast<const uint8_t*>(v_new);
  p.k_cache = static_cast<uint8_t*>(k_cache);
  p.v_cache = static_cast<uint8_t*>(v_cache);
  p.bt = block_table;
  p.seqlens = seqlens;
  p.B = B;
  p.Sk = Sk;
  p.HKV = HKV;
  p.row_bytes = row_bytes;
  p.PS = PS;
  p.BTW = block_table ? BTW : 1;
  p.P = num_pages;
  const long long total = static_cast<long long>(B) * Sk * HKV * (row_bytes / 16);
  long long blocks = (total + 255) / 256;
  if (blocks > 8LL * sm_count()) blocks = 8LL * sm_count();
  kv_append_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("kv_append_kernel");
}

int mxfa_seqlens_add_launch(void* seqlens, int is_int64, int B, int delta, void* stream) {
  if (B < 0 || (B > 0 && seqlens == nullptr)) return fail(MXFA_ERR_INVALID, "invalid seqlens argument");
  if (B == 0 || delta == 0) return MXFA_OK;
  seqlens_add_kernel<<<(B + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(seqlens, is_int64, B, delta);
  return check_launch("seqlens_add_kernel");
}

static int varlen_fwd_impl(const void* q, const void* k, const void* v, const int32_t* cu_q, const int32_t* cu_k,
                           void* out, float* lse, int B, int max_q, int max_k, int total_q, int total_k, int HQ,
                           int HKV, int D, int causal, int bf16, float scale, void* stream, bool exact) {
  if (D != 64 && D != 128) return fail(MXFA_ERR_UNSUPPORTED, "head dim %d not in {64, 128}", D);
  if (B < 0 || max_q < 0 || max_k < 0 || HQ <= 0 || HKV <= 0 || HQ % HKV != 0)
    return fail(MXFA_ERR_INVALID, "bad varlen geometry");
  if ((cu_q == nullptr) != (cu_k == nullptr)) return fail(MXFA_ERR_INVALID, "cu_q and cu_k must both be given");
  if (B == 0 || max_q == 0 || total_q == 0) return MXFA_OK;
  if (total_q < 0 || total_k <= 0) return fail(MXFA_ERR_INVALID, "total token counts must be positive");
  if (cu_q == nullptr && (total_q != static_cast<long long>(B) * max_q || total_k != static_cast<long long>(B) * max_k))
    return fail(MXFA_ERR_INVALID, "dense layout needs total_q = B*max_q and total_k = B*max_k");
  if (!q || !k || !v || !out) return fail(MXFA_ERR_INVALID, "null tensor pointer");
  // the epilogue writes each output row in 16-byte stores
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return fail(MXFA_ERR_INVALID, "tensors must be 16-byte aligned");
  if (HQ > 65535 || B > 65535) return fail(MXFA_ERR_UNSUPPORTED, "grid too large");
  PrefillParams p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.cu_q = cu_q;
  p.cu_k = cu_k;
  p.out = out;
  p.lse = lse;
  p.B = B;
  p.Sq = max_q;
  p.Sk = max_k;
  p.HQ = HQ;
  p.HKV = HKV;
  p.GQ = HQ / HKV;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * kLog2e;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // TMA maps cover exactly the token rows of q and k/v: boxes reaching past
  // the last row read zeros instead of memory beyond the tensors
  int dev = 0;
  cudaGetDevice(&dev);
  const MapKey key{dev, q, k, v, D, HQ, (static_cast<long long>(HKV) << 32) | static_cast<unsigned>(total_q),
                   total_k};
  PrefillMaps maps;
  if (!g_prefill_maps.get(key, &maps)) {
    if (!encode_rows_map(&maps.q, q, D, HQ, total_q, kTcRows) ||
        !encode_rows_map(&maps.k, k, D, HKV, total_k, kTcKeys) ||
        !encode_rows_map(&maps.v, v, D, HKV, total_k, kTcKeys))
      return fail(MXFA_ERR_UNSUPPORTED, "TMA descriptor encoding failed for the prefill operands");
    g_prefill_maps.put(key, maps);
  }
  const CUtensorMap& mq = maps.q;
  const CUtensorMap& mk = maps.k;
  const CUtensorMap& mv = maps.v;
  dim3 grid(HQ, B, (max_q + kTcRows - 1) / kTcRows);
  auto go = [&](auto kern, int smem, std::atomic<unsigned long long>& done, int threads) -> int {
    if (int rc = ensure_smem(kern, smem, done)) return rc;
    kern<<<grid, threads, smem, st>>>(p, mq, mk, mv);
    return check_launch("prefill_tc_kernel");
  };
  static std::atomic<unsigned long long> d0{0}, d1{0}, d2{0}, d3{0}, e0{0}, e1{0}, e2{0}, e3{0};
  if (exact) {
    if (bf16)
      return D == 128
                 ? go(prefill_tc_kernel<__nv_bfloat16, 128, true>, TcCfg<128>::kSmemBytes, e0, TcCfg<128>::kThreads)
                 : go(prefill_tc_kernel<__nv_bfloat16, 64, true>, TcCfg<64>::kSmemBytes, e1, TcCfg<64>::kThreads);
    return D == 128 ? go(prefill_tc_kernel<__half, 128, true>, TcCfg<128>::kSmemBytes, e2, TcCfg<128>::kThreads)
                    : go(prefill_tc_kernel<__half, 64, true>, TcCfg<64>::kSmemBytes, e3, TcCfg<64>::kThreads);
  }
  if (bf16)
    return D == 128 ? go(prefill_tc_kernel<__nv_bfloat16, 128>, TcCfg<128>::kSmemBytes, d0, TcCfg<128>::kThreads)
                    : go(prefill_tc_kernel<__nv_bfloat16, 64>, TcCfg<64>::kSmemBytes, d1, TcCfg<64>::kThreads);
  return D == 128 ? go(prefill_tc_kernel<__half, 128>, TcCfg<128>::kSmemBytes, d2, TcCfg<128>::kThreads)
                  : go(prefill_tc_kernel<__half, 64>, TcCfg<64>::kSmemBytes, d3, TcCfg<64>::kThreads);
}

int mxfa_varlen_fwd_launch(const void* q, const void* k, const void* v, const int32_t* cu_q, const int32_t* cu_k,
                           void* out, float* lse, int B, int max_q, int max_k, int total_q, int total_k, int HQ,
                           int HKV, int D, int causal, int bf16, float scale, void* stream) {
  return varlen_fwd_impl(q, k, v, cu_q, cu_k, out, lse, B, max_q, max_k, total_q, total_k, HQ, HKV, D, causal, bf16,
                         scale, stream, false);
}

int mxfa_varlen_fwd_exact_launch(const void* q, const void* k, const void* v, const int32_t* cu_q,
                                 const int32_t* cu_k, void* out, float* lse, int B, int max_q, int max_k, int total_q,
                                 int total_k, int HQ, int HKV, int D, int causal, int bf16, float scale, void* stream) {
  return varlen_fwd_impl(q, k, v, cu_q, cu_k, out, lse, B, max_q, max_k, total_q, total_k, HQ, HKV, D, causal, bf16,
                         scale, stream, true);
}


}  // extern "C"

// ------------------------------------------------------- allocation-free variant
//
// Some callers cannot allocate device memory at the point where they run
// attention: an inference engine that reserved the whole GPU for its own KV
// pool up front, a host runtime reaching this library through a plain C FFI
// with no device allocator of its own, or a latency-critical loop where a
// cudaMalloc (which may synchronise the device) is not acceptable.  For them
// the split partials live in one fixed buffer compiled into the library.
//
// The buffer is a file-scope __device__ array, so every GPU that loads the
// library holds MXFA_NOALLOC_SCRATCH_BYTES of it until the process exits.
// Its name is only a host-side stand-in: the device address is obtained with
// cudaGetSymbolAddress with the device current, on the first call made on
// that device, and again whenever that device's context has changed since
// (a cudaDeviceReset tears the module down, and the re-created context may
// place the array elsewhere).  All calls on a device share the buffer and
// leave their partials in it; nothing needs to start at zero because the
// decode kernel writes every partial slot the combine kernel then reads.
namespace mxfa {
namespace {

static __device__ __align__(256) float g_noalloc_scratch[MXFA_NOALLOC_SCRATCH_BYTES / sizeof(float)];

// Process-unique id of the calling thread's current context (0 if none or
// the driver cannot say).  Context ids are never reused within a process,
// unlike context handles.
unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(p);
    p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(p);
  });
  if (get_current == nullptr || get_id == nullptr) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

int noalloc_scratch(float** out) {
  static float* addr[64] = {};
  static unsigned long long ctx_id[64] = {};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(MXFA_ERR_CUDA, "cudaGetDevice failed: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(MXFA_ERR_UNSUPPORTED, "device index %d out of range", dev);
  const unsigned long long id = current_context_id();
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr || id == 0 || id != ctx_id[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(MXFA_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed on device %d: %s", dev,
                  cudaGetErrorString(e));
    addr[dev] = static_cast<float*>(p);
    // the lookup makes the device's context current if nothing was yet
    ctx_id[dev] = current_context_id();
  }
  *out = addr[dev];
  return MXFA_OK;
}

}  // namespace
}  // namespace mxfa

extern "C" int mxfa_kvcache_attention_noalloc_launch(const void* q, const void* k_cache, const void* v_cache,
                                                     const int32_t* block_table, const int32_t* seqlens, void* out,
                                                     float* lse, int B, int Sq, int HQ, int HKV, int D, int PS,
                                                     int BTW, int num_pages, int append_len, int num_splits,
                                                     int chunk_len, int causal, int bf16, float scale,
                                                     void* stream) {
  // The same argument checks as the workspace entry point, first, so a bad
  // argument is reported as itself and never as a scratch-size refusal.
  if (D != 64 && D != 128) return fail(MXFA_ERR_UNSUPPORTED, "head dim %d not in {64, 128}", D);
  if (B < 0 || Sq < 0 || HQ <= 0 || HKV <= 0 || HQ % HKV != 0)
    return fail(MXFA_ERR_INVALID, "bad head / batch geometry (B=%d Sq=%d HQ=%d HKV=%d)", B, Sq, HQ, HKV);
  if (B == 0 || Sq == 0) return MXFA_OK;
  if (PS <= 0 || num_pages <= 0 || append_len < 0) return fail(MXFA_ERR_INVALID, "bad cache geometry");
  if (block_table != nullptr && BTW <= 0) return fail(MXFA_ERR_INVALID, "block table width must be positive");
  if (!q || !k_cache || !v_cache || !seqlens || !out) return fail(MXFA_ERR_INVALID, "null tensor pointer");
  const long long rows = static_cast<long long>(B) * Sq * HQ;
  if (rows > 0x7FFFFFFFll) return fail(MXFA_ERR_UNSUPPORTED, "%lld query rows exceed the 32-bit row index", rows);
  int max_len = 0;
  if (int rc = cache_capacity(block_table, BTW, PS, &max_len)) return rc;
  if (num_splits <= 0 || chunk_len <= 0) mxfa_kvcache_plan(B, Sq, HQ, HKV, D, max_len, &num_splits, &chunk_len);
  float* scratch = nullptr;
  if (num_splits > 1) {
    const size_t need = mxfa_split_workspace_bytes(static_cast<int>(rows), D, num_splits);
    if (need > MXFA_NOALLOC_SCRATCH_BYTES)
      return fail(MXFA_ERR_UNSUPPORTED,
                  "allocation-free call needs %zu bytes of split scratch but the built-in buffer holds %u; "
                  "use fewer splits or a smaller batch, or mxfa_kvcache_attention_launch with a caller workspace",
                  need, static_cast<unsigned>(MXFA_NOALLOC_SCRATCH_BYTES));
    if (int rc = noalloc_scratch(&scratch)) return rc;
  }
  return mxfa_kvcache_attention_launch(q, k_cache, v_cache, block_table, seqlens, out, lse, scratch,
                                       scratch ? MXFA_NOALLOC_SCRATCH_BYTES : 0, B, Sq, HQ, HKV, D, PS, BTW,
                                       num_pages, append_len, num_splits, chunk_len, causal, bf16, scale, stream);
}
