// attn_bwd_b200.cu — C-ABI entry points: argument checks, TMA descriptors,
// launches of the fused dS and dV kernels on the caller's stream.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>

#include "../../include/attn_bwd_b200.h"
#include "ds_kernel.cuh"
#include "dv_kernel.cuh"

using namespace attn_bwd;

namespace {

__device__ int g_kernel_error = 0;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

constexpr int kMaxDevices = 64;
struct DeviceState {
  bool ready = false;
  int rc = ATTN_BWD_OK;
  int sm_count = 0;
  int* err = nullptr;  // device address of g_kernel_error on this device
  // Side stream + fork/join events for running the dV kernel next to the dS kernel
  // (created once per device, on the first full call; never destroyed).
  cudaStream_t side = nullptr;
  // cudaOccupancyMaxActiveClusters per (dS kernel instance, cluster size), filled on first use
  struct OccEntry { const void* kern; int cs; int clusters; };
  OccEntry occ[32] = {};
  int n_occ = 0;
  cudaEvent_t fork = nullptr, join = nullptr;
  std::mutex side_mu;   // one full call at a time uses the side stream
  // Full calls replayed as CUDA graphs, keyed by their whole argument list (16-entry LRU).
  struct GraphEntry {
    uint64_t key[14];
    int state;             // 0 empty, 1 seen once (ran eagerly), 2 graph ready
    uint64_t last_use;
    cudaGraphExec_t exec;
  };
  GraphEntry graphs[16] = {};
  uint64_t graph_clock = 0;
  cudaStream_t cap = nullptr;   // private stream the captures run on
  // Host-buffer calls (attn_bwd_b200_host_shard): copy-in and copy-out streams and the
  // per-chunk events between the three stages (created on first use; never destroyed).
  std::mutex host_mu;   // one host-buffer call at a time enqueues on these
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t h_fork = nullptr, h_join = nullptr;
  cudaEvent_t in_done[64] = {}, comp_done[64] = {};
};
std::mutex g_mu;
DeviceState g_dev[kMaxDevices];

// Measurement / test options (attn_bwd_b200_set_option).  Process-wide; every call reads
// them when it chooses its kernels; the generation counter is part of the launch-graph key,
// so a change never replays a graph recorded under other options.
constexpr int kNumOptions = ATTN_BWD_OPT_COUNT;
std::atomic<int> g_opt[kNumOptions];
std::atomic<unsigned> g_opt_gen{0};
struct OptDefaults {
  OptDefaults() {
    for (int i = 0; i < kNumOptions; ++i) g_opt[i].store(-1);
  }
} g_opt_defaults;
inline int opt(int k) { return g_opt[k].load(std::memory_order_relaxed); }
EncodeTiledFn g_encode = nullptr;

bool set_ds_smem() {
#define ATTN_BWD_SMEM(R, M)                                                                               \
  (cudaFuncSetAttribute(ds::ds_kernel<R, M>, cudaFuncAttributeMaxDynamicSharedMemorySize,                 \
                        ds::Cfg<R, M>::SMEM_BYTES) == cudaSuccess)
  return ATTN_BWD_SMEM(ds::kRowsAligned, ds::kRecompute) && ATTN_BWD_SMEM(ds::kRowsAligned, ds::kResident) &&
         ATTN_BWD_SMEM(ds::kRowsAligned, ds::kTmemP) && ATTN_BWD_SMEM(ds::kRowsAligned, ds::kCompact) &&
         ATTN_BWD_SMEM(ds::kRowsRagged, ds::kRecompute) && ATTN_BWD_SMEM(ds::kRowsRagged, ds::kResident) &&
         ATTN_BWD_SMEM(ds::kRowsRagged, ds::kTmemP) && ATTN_BWD_SMEM(ds::kRowsClass, ds::kRecompute) &&
         ATTN_BWD_SMEM(ds::kRowsClass, ds::kResident) && ATTN_BWD_SMEM(ds::kRowsClass, ds::kTmemP) &&
         ATTN_BWD_SMEM(ds::kRowsClass, ds::kCompact);
#undef ATTN_BWD_SMEM
}

int device_state(DeviceState** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return ATTN_BWD_ECUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& st = g_dev[dev];
  if (!st.ready) {
    st.ready = true;
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
      st.rc = ATTN_BWD_ECUDA;
    } else if (major != 10) {
      st.rc = ATTN_BWD_EDEVICE;
    } else if (cudaDeviceGetAttribute(&st.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
               !set_ds_smem() ||
               cudaFuncSetAttribute(dv::dv_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    dv::Cfg<false>::SMEM_BYTES) != cudaSuccess ||
               cudaFuncSetAttribute(dv::dv_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    dv::Cfg<true>::SMEM_BYTES) != cudaSuccess ||
               cudaFuncSetAttribute(dv::dv_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    dv::Cfg<false, true>::SMEM_BYTES) != cudaSuccess ||
               cudaGetSymbolAddress(reinterpret_cast<void**>(&st.err), g_kernel_error) != cudaSuccess) {
      st.rc = ATTN_BWD_ECUDA;
    }
    if (st.rc == ATTN_BWD_OK && !g_encode) {
      cudaDriverEntryPointQueryResult q;
      void* fn = nullptr;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
          q != cudaDriverEntryPointSuccess || !fn) {
        st.rc = ATTN_BWD_ETMAP;
      } else {
        g_encode = reinterpret_cast<EncodeTiledFn>(fn);
      }
    }
  }
  *out = &st;
  return st.rc;
}

bool encode_map(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* ptr, const cuuint64_t* dims,
                const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle sw) {
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode(m, dt, rank, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Encoded descriptors, direct-mapped by a hash of every encode argument (a descriptor
// depends on nothing else), so repeated calls on the same tensors skip the driver call.
// Option ATTN_BWD_OPT_MAP_CACHE = 0 encodes every time.
struct MapEntry {
  uint64_t key[16];
  bool valid;
  CUtensorMap map;
};
constexpr int kMapCacheSize = 256;
MapEntry g_maps[kMapCacheSize];
std::mutex g_map_mu;

bool make_map(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* ptr, const cuuint64_t* dims,
              const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle sw) {
  const bool cache_on = opt(ATTN_BWD_OPT_MAP_CACHE) != 0;
  if (!cache_on || rank > 5) return encode_map(m, dt, rank, ptr, dims, strides, box, sw);
  uint64_t key[16] = {};
  key[0] = (uint64_t)dt | ((uint64_t)rank << 8) | ((uint64_t)sw << 16);
  key[1] = (uint64_t)reinterpret_cast<uintptr_t>(ptr);
  for (int i = 0; i < rank; ++i) {
    key[2 + i] = dims[i];
    key[7 + i] = box[i];
    if (i + 1 < rank) key[12 + i] = strides[i];
  }
  uint64_t h = 1469598103934665603ull;   // FNV-1a over the key words
  for (uint64_t w : key) h = (h ^ w) * 1099511628211ull;
  MapEntry& e = g_maps[h % kMapCacheSize];
  {
    std::lock_guard<std::mutex> lk(g_map_mu);
    if (e.valid && std::memcmp(e.key, key, sizeof(key)) == 0) {
      *m = e.map;
      return true;
    }
  }
  if (!encode_map(m, dt, rank, ptr, dims, strides, box, sw)) return false;
  std::lock_guard<std::mutex> lk(g_map_mu);
  std::memcpy(e.key, key, sizeof(key));
  e.map = *m;
  e.valid = true;
  return true;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct Shape {
  int bs, sq, skv, u0, u1;
  int n_units() const { return u1 - u0; }
  // element counts of the shard's tensors (a null pointer is accepted only for an empty one)
  long long n_scores() const { return (long long)n_units() * kGroups * sq * skv; }
  long long n_dO() const { return (long long)bs * sq * kHeads * kHeadDim; }
  long long n_V() const { return (long long)bs * kKvHeads * skv * kHeadDim; }
  long long n_dV() const { return (long long)n_units() * skv * kHeadDim; }
};

inline bool ptr_ok(const void* p, long long n) { return p != nullptr || n == 0; }

int check_shape(const Shape& s) {
  if (s.bs < 0 || s.sq < 0 || s.skv < 0) return ATTN_BWD_EINVAL;
  if (s.u0 < 0 || s.u1 < s.u0 || s.u1 > s.bs * kKvHeads) return ATTN_BWD_EINVAL;
  // TMA descriptor limits: every extent < 2^31 and strides < 2^40 bytes
  const long long rows = (long long)s.bs * kHeads * s.sq;
  if ((long long)s.sq * s.skv * 2 >= (1ll << 39) || rows * s.skv >= (1ll << 40) || s.sq >= (1 << 30) ||
      s.skv >= (1 << 30))
    return ATTN_BWD_EINVAL;
  return ATTN_BWD_OK;
}

// Pass-2 mode of the dS kernel, chosen per shape from B200 measurements (clusters cost:
// forcing c1 onto 2-CTA clusters made its dS kernel 27 % slower, so the modes that keep a
// row in one CTA come first):
//   ragged rows: kTmemP while a row fits 5 chunks per CTA on clusters of up to 8
//     CTAs (its pass 2 avoids re-fetching unaligned rows: c2 dS 553 -> 348 us);
//   aligned rows: kResident up to 8 chunks (6 shared P/mask stages beat kTmemP's 4
//     dedicated ones: c1 100 vs 120 us), kCompact for 9-10 chunks (one CTA instead of a
//     cluster), kResident on clusters beyond that;
//   then kResident on clusters up to 8 x 512 columns, then kRecompute.
// Option ATTN_BWD_OPT_DS_MODE = 0/1/2/3 forces recompute / resident / TMEM-P / compact
// where the shape allows it (measurements and tests).
int forced_ds_mode() { return opt(ATTN_BWD_OPT_DS_MODE); }

// seq_kv rows of P / mask / dS must be 16-byte multiples for the TMA path.
inline bool tma_rows_ok(int skv) { return (skv % 16) == 0; }

// dv_units_of: CTAs the dV kernel launches for this shape (min(units, SMs)).
int dv_ctas(const DeviceState& st, const Shape& s) {
  if (s.n_units() == 0 || s.skv == 0 || s.sq == 0) return 0;
  const int units = s.n_units() * ((s.skv + dv::BM - 1) / dv::BM);
  return units < st.sm_count ? units : st.sm_count;
}

int launch_ds(const DeviceState& st, const Shape& s, const void* dO, const void* P, const void* V,
              const uint8_t* M, float p, void* dS, cudaStream_t stream, int max_ctas = 0) {
  const int nbh = s.n_units() * kGroups;
  if (nbh == 0 || s.sq == 0 || s.skv == 0) return ATTN_BWD_OK;
  // Rows whose length is not a multiple of 16 bytes: class tiles (16·64 rows per tile set)
  // unless they need over 10 % more row slots than 128-row blocks per head do, else the
  // per-row re-aligning kernel.  Measured on B200 (dS us, class / per-row; slot ratio):
  // c2 243 / 339 (0.80), 32x691x773 2264 / 3730 (0.93), 8x373x449 212 / 240 (1.07),
  // 4x211x293 76 / 62 (1.20).
  // Option ATTN_BWD_OPT_ROW_KIND = 1 (per-row) / 2 (class tiles) forces one of the two (the
  // latter also for aligned rows, as a measurement of the class layout alone).
  const bool force_ragged = opt(ATTN_BWD_OPT_ROW_KIND) == 1;
  const bool force_class = opt(ATTN_BWD_OPT_ROW_KIND) == 2;
  const bool rag = !tma_rows_ok(s.skv);
  int rk = ds::kRowsAligned;
  if (rag || force_class) {
    const long long per_class = (kGroups * (long long)s.sq + 15) / 16;
    const long long class_slots = (per_class + 63) / 64 * 64 * 16;
    const long long block_slots = (long long)kGroups * ((s.sq + ds::BM - 1) / ds::BM) * ds::BM;
    rk = (force_class || (!force_ragged && class_slots * 10 <= block_slots * 11)) ? ds::kRowsClass : ds::kRowsRagged;
  }
  const long long total_rows = (long long)nbh * s.sq;
  const long long cls_y = rk == ds::kRowsClass ? total_rows / 16 : 0;
  CUtensorMap tm_dO, tm_V, tm_P, tm_M, tm_dS;
  std::memset(&tm_P, 0, sizeof(tm_P));
  std::memset(&tm_M, 0, sizeof(tm_M));
  std::memset(&tm_dS, 0, sizeof(tm_dS));
  {
    cuuint64_t dims[4] = {kHeadDim, kHeads, (cuuint64_t)s.sq, (cuuint64_t)s.bs};
    cuuint64_t str[3] = {kHeadDim * 2, (cuuint64_t)kHeads * kHeadDim * 2, (cuuint64_t)s.sq * kHeads * kHeadDim * 2};
    cuuint32_t box[4] = {64, 1, ds::BM, 1};
    if (!make_map(&tm_dO, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, dO, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return ATTN_BWD_ETMAP;
  }
  {
    cuuint64_t dims[3] = {kHeadDim, (cuuint64_t)s.skv, (cuuint64_t)s.bs * kKvHeads};
    cuuint64_t str[2] = {kHeadDim * 2, (cuuint64_t)s.skv * kHeadDim * 2};
    cuuint32_t box[3] = {64, ds::BN, 1};
    if (!make_map(&tm_V, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, V, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return ATTN_BWD_ETMAP;
  }
  if (!rag) {
    cuuint64_t dims[3] = {(cuuint64_t)s.skv, (cuuint64_t)s.sq, (cuuint64_t)nbh};
    cuuint64_t str2[2] = {(cuuint64_t)s.skv * 2, (cuuint64_t)s.sq * s.skv * 2};
    cuuint64_t str1[2] = {(cuuint64_t)s.skv, (cuuint64_t)s.sq * s.skv};
    cuuint32_t box[3] = {ds::BN, ds::BM, 1};
    if (!make_map(&tm_P, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, P, dims, str2, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map(&tm_dS, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dS, dims, str2, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map(&tm_M, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, M, dims, str1, box, CU_TENSOR_MAP_SWIZZLE_64B))
      return ATTN_BWD_ETMAP;
  }
  if (cls_y > 0) {
    // class rows: the local P / mask buffers as 16-row groups, 16·skv elements each; a box
    // is 64 rows of one class (64 groups) x one 64-column window
    cuuint64_t dims[2] = {(cuuint64_t)s.skv * 16, (cuuint64_t)cls_y};
    cuuint64_t str2[1] = {(cuuint64_t)s.skv * 32};
    cuuint64_t str1[1] = {(cuuint64_t)s.skv * 16};
    cuuint32_t boxp[2] = {ds::BN, 64};
    cuuint32_t boxm[2] = {ds::CLS_M_PITCH, 64};
    if (!make_map(&tm_P, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, P, dims, str2, boxp, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map(&tm_dS, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dS, dims, str2, boxp, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map(&tm_M, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, M, dims, str1, boxm, CU_TENSOR_MAP_SWIZZLE_NONE))
      return ATTN_BWD_ETMAP;
  }
  ds::Params prm;
  prm.sq = s.sq;
  prm.skv = s.skv;
  if (rk == ds::kRowsClass) {
    // units: (kv group, class pair, 64-row tile); a window starts up to 7 columns early
    const int per_class = (kGroups * s.sq + 15) / 16;
    prm.cls_T = (per_class + 63) / 64;
    prm.cls_Y = (int)cls_y;
    prm.n_mb = 1;
    prm.n_units = s.n_units() * 8 * prm.cls_T;
    prm.nchunks = (s.skv + 7 + ds::BN - 1) / ds::BN;
  } else {
    prm.cls_T = 1;
    prm.cls_Y = 0;
    prm.n_mb = (s.sq + ds::BM - 1) / ds::BM;
    prm.n_units = nbh * prm.n_mb;
    prm.nchunks = (s.skv + ds::BN - 1) / ds::BN;
  }
  prm.dO = static_cast<const uint8_t*>(dO);
  // Rows that do not fit one CTA's TMEM plan are split over a cluster of cs <= 8
  // CTAs (CTA k owns chunks [k*cpc, (k+1)*cpc)); the CTAs exchange row sums.
  auto split = [&](int per_cta) {
    prm.cs = (prm.nchunks + per_cta - 1) / per_cta;
    prm.cpc = (prm.nchunks + prm.cs - 1) / prm.cs;
  };
  const int tp_max = ds::Cfg<ds::kRowsAligned, ds::kTmemP>::NSLOT;
  const int cp_max = ds::Cfg<ds::kRowsAligned, ds::kCompact>::CP_MAX;
  const int forced = forced_ds_mode();
  int mode;
  // per-row re-aligned rows: kTmemP; aligned and class rows: kResident measured faster
  const bool tp_pref = rk == ds::kRowsRagged ? prm.nchunks <= 8 * tp_max : false;
  if ((forced < 0 && tp_pref) || (forced == ds::kTmemP && prm.nchunks <= 8 * tp_max)) {
    mode = ds::kTmemP;
    split(tp_max);
  } else if (rk != ds::kRowsRagged && ((forced < 0 && prm.nchunks > ds::TSLOTS && prm.nchunks <= cp_max) ||
                      (forced == ds::kCompact && prm.nchunks <= 8 * cp_max))) {
    // 9-10 chunks: the bf16 compact store keeps the row in one CTA (c4 dS 1966 -> 1643 us);
    // where a cluster is needed anyway, kResident's exact fp32 store measured faster
    // (c3 1187 vs 1343 us), so kCompact is not used there
    mode = ds::kCompact;
    split(cp_max);
  } else if (prm.nchunks <= 8 * ds::TSLOTS && forced != ds::kRecompute) {
    mode = ds::kResident;
    split(ds::TSLOTS);
    // option ATTN_BWD_OPT_DS_CLUSTER = n forces n CTAs per row (1..8) when it fits
    const int forced_cs = opt(ATTN_BWD_OPT_DS_CLUSTER);
    if (forced_cs >= 1 && forced_cs <= 8 && (prm.nchunks + forced_cs - 1) / forced_cs <= ds::TSLOTS &&
        forced_cs <= prm.nchunks) {
      prm.cs = forced_cs;
      prm.cpc = (prm.nchunks + forced_cs - 1) / forced_cs;
    }
  } else {
    mode = ds::kRecompute;
    prm.cs = 1;
    prm.cpc = prm.nchunks;
  }
  prm.resident = mode != ds::kRecompute;
  prm.bh_base = s.u0 * kGroups;
  prm.use_mask = p > 0.f ? 1 : 0;
  // L2 prefetch of a CTA's next unit during pass 2 (aligned rows only): measured on B200
  // over the SOL-ExecBench shapes and c1-c4, it helps rows of up to 6 chunks held by one
  // CTA (c1 dS 97 -> 91 us, 64x128x128 161 -> 155 us) and hurts longer rows (c4 dS
  // 2010 -> 2096 us, 1x4096x4096 +5 %), where the extra L2 footprint evicts pass-2 data.
  // Option ATTN_BWD_OPT_L2_PREFETCH = 0/1 forces it off / on (measurements).
  const int l2pf_env = opt(ATTN_BWD_OPT_L2_PREFETCH);
  prm.l2pf = l2pf_env >= 0 ? l2pf_env : (prm.cs == 1 && prm.nchunks <= 6 ? 1 : 0);
  // L2 eviction hints on the aligned path (pass-1 P / mask kept for pass 2, pass-2 reloads
  // and dS stores evicted first): measured on B200, c3 dS 1279 -> 1245 us, c1 96 -> 91 us,
  // c4 unchanged.  Option ATTN_BWD_OPT_L2_HINT = 0 turns them off (measurements).
  const int l2hint_env = opt(ATTN_BWD_OPT_L2_HINT) < 0 ? 1 : opt(ATTN_BWD_OPT_L2_HINT);
  // class rows: option value 2 (measurement) also applies them there
  prm.l2hint = rk == ds::kRowsClass ? (l2hint_env == 2 ? 1 : 0) : (l2hint_env != 0 ? 1 : 0);
  prm.scale = p > 0.f ? 1.0f / (1.0f - p) : 1.0f;
  prm.err = st.err;
  prm.P = static_cast<const uint8_t*>(P);
  prm.M = M;
  prm.dS = static_cast<uint8_t*>(dS);
  const unsigned long long E = (unsigned long long)nbh * s.sq * s.skv;
  prm.p_end16 = (E * 2 + 15) & ~15ull;
  prm.m_end16 = (E + 15) & ~15ull;

  void (*kern)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
               const ds::Params) = nullptr;
  int smem = 0;
#define ATTN_BWD_PICK(R, M)                    \
  if (rk == R && mode == M) {                  \
    kern = ds::ds_kernel<R, M>;                \
    smem = ds::Cfg<R, M>::SMEM_BYTES;          \
  }
  ATTN_BWD_PICK(ds::kRowsAligned, ds::kRecompute)
  ATTN_BWD_PICK(ds::kRowsAligned, ds::kResident)
  ATTN_BWD_PICK(ds::kRowsAligned, ds::kTmemP)
  ATTN_BWD_PICK(ds::kRowsAligned, ds::kCompact)
  ATTN_BWD_PICK(ds::kRowsRagged, ds::kRecompute)
  ATTN_BWD_PICK(ds::kRowsRagged, ds::kResident)
  ATTN_BWD_PICK(ds::kRowsRagged, ds::kTmemP)
  ATTN_BWD_PICK(ds::kRowsClass, ds::kRecompute)
  ATTN_BWD_PICK(ds::kRowsClass, ds::kResident)
  ATTN_BWD_PICK(ds::kRowsClass, ds::kTmemP)
  ATTN_BWD_PICK(ds::kRowsClass, ds::kCompact)
#undef ATTN_BWD_PICK
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.blockDim = dim3(ds::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  const int sm_budget = (max_ctas > 0 && max_ctas < st.sm_count) ? max_ctas : st.sm_count;
  int clusters = sm_budget;
  if (prm.cs > 1) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = prm.cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(prm.cs * st.sm_count);
    int max_clusters = 0;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      DeviceState& mst = const_cast<DeviceState&>(st);
      for (int i = 0; i < mst.n_occ; ++i)
        if (mst.occ[i].kern == (const void*)kern && mst.occ[i].cs == prm.cs) max_clusters = mst.occ[i].clusters;
      if (!max_clusters) {
        if (cudaOccupancyMaxActiveClusters(&max_clusters, kern, &cfg) != cudaSuccess || max_clusters < 1)
          return ATTN_BWD_ECUDA;
        if (mst.n_occ < 32) mst.occ[mst.n_occ++] = {(const void*)kern, prm.cs, max_clusters};
      }
    }
    clusters = max_clusters;
    if (clusters * prm.cs > sm_budget) clusters = sm_budget / prm.cs > 0 ? sm_budget / prm.cs : 1;
  }
  const int n_clusters = prm.n_units < clusters ? prm.n_units : clusters;
  cfg.gridDim = dim3(n_clusters * prm.cs);
  if (cudaLaunchKernelEx(&cfg, kern, tm_dO, tm_V, tm_P, tm_M, tm_dS, prm) != cudaSuccess) return ATTN_BWD_ECUDA;
  return cudaPeekAtLastError() == cudaSuccess ? ATTN_BWD_OK : ATTN_BWD_ECUDA;
}

// Pd is attn_weights_dropped; or, with M != nullptr, attn_weights, and the kernel forms
// P_drop = bf16(P * M / (1-p)) itself (seq_kv % 16 == 0 only).
int launch_dv(const DeviceState& st, const Shape& s, const void* dO, const void* Pd, void* dV,
              cudaStream_t stream, int max_ctas = 0, const uint8_t* M = nullptr, float p = 0.f) {
  const bool fpm = M != nullptr;
  const int nu = s.n_units();
  if (nu == 0 || s.skv == 0) return ATTN_BWD_OK;
  if (s.sq == 0) {  // empty sum over seq_q: dV = 0
    const size_t bytes = (size_t)nu * s.skv * kHeadDim * 2;
    return cudaMemsetAsync(dV, 0, bytes, stream) == cudaSuccess ? ATTN_BWD_OK : ATTN_BWD_ECUDA;
  }
  // P_drop rows need only be 16-byte multiples (seq_kv % 8) for the TMA path
  const bool rag = (s.skv % 8) != 0;
  if (fpm && rag) return ATTN_BWD_EUNSUPPORTED;
  CUtensorMap tm_Pd, tm_dO, tm_M;
  std::memset(&tm_Pd, 0, sizeof(tm_Pd));
  std::memset(&tm_M, 0, sizeof(tm_M));
  if (fpm) {
    if (s.skv % 16) return ATTN_BWD_EUNSUPPORTED;   // mask rows must be 16-byte multiples for TMA
    cuuint64_t dims[3] = {(cuuint64_t)s.skv, (cuuint64_t)s.sq, (cuuint64_t)nu * kGroups};
    cuuint64_t str[2] = {(cuuint64_t)s.skv, (cuuint64_t)s.sq * s.skv};
    cuuint32_t box[3] = {dv::BM, dv::BK, 1};
    if (!make_map(&tm_M, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, M, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return ATTN_BWD_ETMAP;
  }
  if (!rag) {
    cuuint64_t dims[3] = {(cuuint64_t)s.skv, (cuuint64_t)s.sq, (cuuint64_t)nu * kGroups};
    cuuint64_t str[2] = {(cuuint64_t)s.skv * 2, (cuuint64_t)s.sq * s.skv * 2};
    cuuint32_t box[3] = {64, dv::BK, 1};
    if (!make_map(&tm_Pd, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, Pd, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return ATTN_BWD_ETMAP;
  }
  // ragged rows: every 8th row is 16·skv bytes further, so rows of one class mod 8 form a
  // 2-D tensor of 32-bit words (4·skv words per 8-row group) read as 8-row x 272 B boxes
  const long long rows8 = rag ? (long long)nu * kGroups * s.sq / 8 : 0;
  if (rows8 > 0) {
    cuuint64_t dims[2] = {(cuuint64_t)s.skv * 4, (cuuint64_t)rows8};
    cuuint64_t str[1] = {(cuuint64_t)s.skv * 16};
    cuuint32_t box[2] = {dv::Cfg<true>::RAW_PITCH / 4, 8};
    if (!make_map(&tm_Pd, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, Pd, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE))
      return ATTN_BWD_ETMAP;
  }
  {
    cuuint64_t dims[4] = {kHeadDim, kHeads, (cuuint64_t)s.sq, (cuuint64_t)s.bs};
    cuuint64_t str[3] = {kHeadDim * 2, (cuuint64_t)kHeads * kHeadDim * 2, (cuuint64_t)s.sq * kHeads * kHeadDim * 2};
    cuuint32_t box[4] = {64, 1, dv::BK, 1};
    if (!make_map(&tm_dO, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, dO, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return ATTN_BWD_ETMAP;
  }
  dv::Params prm;
  prm.sq = s.sq;
  prm.skv = s.skv;
  prm.n_jt = (s.skv + dv::BM - 1) / dv::BM;
  prm.n_units = nu * prm.n_jt;
  prm.n_kc = (s.sq + dv::BK - 1) / dv::BK;
  prm.unit_base = s.u0;
  prm.err = st.err;
  prm.Pd = static_cast<const uint8_t*>(Pd);
  prm.pd_end16 = ((unsigned long long)nu * kGroups * s.sq * s.skv * 2 + 15) & ~15ull;
  prm.tma_rows = rows8 * 8;
  prm.scale = fpm ? 1.0f / (1.0f - p) : 1.0f;
  int grid = prm.n_units < st.sm_count ? prm.n_units : st.sm_count;
  if (max_ctas > 0 && grid > max_ctas) grid = max_ctas;
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(dV);
  if (rag)
    dv::dv_kernel<true><<<grid, dv::Cfg<true>::kThreads, dv::Cfg<true>::SMEM_BYTES, stream>>>(tm_Pd, tm_dO, out, prm,
                                                                                            tm_M);
  else if (fpm)
    dv::dv_kernel<false, true><<<grid, dv::Cfg<false, true>::kThreads, dv::Cfg<false, true>::SMEM_BYTES, stream>>>(
        tm_Pd, tm_dO, out, prm, tm_M);
  else
    dv::dv_kernel<false><<<grid, dv::Cfg<false>::kThreads, dv::Cfg<false>::SMEM_BYTES, stream>>>(tm_Pd, tm_dO, out, prm,
                                                                                             tm_M);
  return cudaPeekAtLastError() == cudaSuccess ? ATTN_BWD_OK : ATTN_BWD_ECUDA;
}

// Self-test of the bounded-wait machinery: one warp waits on an mbarrier that
// nothing will ever arrive on, with a limit of `limit_ns`.  The wait must give
// up, record `code` in the error flag and let the kernel exit normally.
__global__ void wait_timeout_selftest(int* err, int code, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);
    abort_flag = 0;
    sm100::fence_barrier_init();
  }
  __syncthreads();
  const bool ok = sm100::mbar_wait(&bar, 0, &abort_flag, err, code, limit_ns);
  (void)__all_sync(0xffffffffu, ok);
}

int prologue(DeviceState** st, const Shape& s) {
  int rc = check_shape(s);
  if (rc) return rc;
  return device_state(st);
}


// Issues the dS and dV kernels of one full call on stream cs (see attn_bwd_b200_shard).
// fpm: the dV kernel forms P_drop from P and the mask (Pd unused).
int enqueue_full_locked(DeviceState* st, const Shape& s, const void* dO, const void* P, const void* Pd, const void* V,
                 const uint8_t* M, float p, void* dS, void* dV, cudaStream_t cs, bool fpm = false) {
  const void* dv_src = fpm ? P : Pd;
  const uint8_t* dv_mask = fpm ? M : nullptr;
  int rc = ATTN_BWD_OK;
  // The dS and dV kernels are independent (different inputs and outputs), so the dV
  // kernel always runs on a side stream forked from the caller's stream, which waits for
  // both at the end.  Two forms, chosen from B200 measurements over the SOL-ExecBench
  // shapes and the benchmark configs:
  //   split  (up to 256M score elements; ragged rows: 64M): dV is launched first on a
  //          fixed share of the SMs (32 of 148; ragged rows 48) and runs persistently
  //          next to a dS grid sized to the rest.  Both kernels are latency-bound at
  //          these sizes and overlap well (64x128x128: 178 -> 143 us, 8x128x128:
  //          37 -> 31 us);
  //   plain  (larger): dS is launched first with the full grid and dV's CTAs take over
  //          SMs as dS CTAs finish, filling the dS kernel's tail (1x4096x4096: 2306 us
  //          back to back -> 1979 us).
  // Option ATTN_BWD_OPT_SIDE_STREAM = 0 runs them back to back on one stream.
  const int dvc = dv_ctas(*st, s);
  const bool rag_rows = !tma_rows_ok(s.skv);
  const double elems = (double)s.n_units() * kGroups * s.sq * s.skv;
  const bool small = elems <= (rag_rows ? 64e6 : 256e6);
  const int dv_share = (st->sm_count * (rag_rows ? 48 : 32) + 147) / 148;
  const bool side_on = opt(ATTN_BWD_OPT_SIDE_STREAM) != 0;
  if (side_on && dvc > 0) {
    if (!st->side) {
      if (cudaStreamCreateWithFlags(&st->side, cudaStreamNonBlocking) != cudaSuccess ||
          cudaEventCreateWithFlags(&st->fork, cudaEventDisableTiming) != cudaSuccess ||
          cudaEventCreateWithFlags(&st->join, cudaEventDisableTiming) != cudaSuccess)
        return ATTN_BWD_ECUDA;
    }
    // options ATTN_BWD_OPT_SPLIT = 0/1 force the plain / split form, ATTN_BWD_OPT_DV_SMS = n
    // sets the dV share of the split form (measurements)
    const int force_split = opt(ATTN_BWD_OPT_SPLIT);
    const int dv_sms = opt(ATTN_BWD_OPT_DV_SMS);
    int dv_grid = dv_sms > 0 ? dv_sms : dv_share;
    if (dv_grid > dvc) dv_grid = dvc;
    const int budget = st->sm_count - dv_grid;
    const bool split = budget > 0 && (force_split >= 0 ? force_split == 1 : small);
    int rc_ds = ATTN_BWD_OK, rc_dv = ATTN_BWD_OK;
    if (cudaEventRecord(st->fork, cs) != cudaSuccess || cudaStreamWaitEvent(st->side, st->fork, 0) != cudaSuccess)
      return ATTN_BWD_ECUDA;
    if (split) {
      rc_dv = launch_dv(*st, s, dO, dv_src, dV, st->side, dv_grid, dv_mask, p);
      if (rc_dv == ATTN_BWD_OK) rc_ds = launch_ds(*st, s, dO, P, V, M, p, dS, cs, budget);
    } else {
      rc_ds = launch_ds(*st, s, dO, P, V, M, p, dS, cs);
      if (rc_ds == ATTN_BWD_OK) rc_dv = launch_dv(*st, s, dO, dv_src, dV, st->side, 0, dv_mask, p);
    }
    // join even after an error, so the caller's stream never runs ahead of issued work
    if (cudaEventRecord(st->join, st->side) != cudaSuccess || cudaStreamWaitEvent(cs, st->join, 0) != cudaSuccess)
      return ATTN_BWD_ECUDA;
    return rc_ds ? rc_ds : rc_dv;
  }
  rc = launch_ds(*st, s, dO, P, V, M, p, dS, cs);
  if (rc) return rc;
  return launch_dv(*st, s, dO, dv_src, dV, cs, 0, dv_mask, p);
}


int enqueue_full(DeviceState* st, const Shape& s, const void* dO, const void* P, const void* Pd, const void* V,
                 const uint8_t* M, float p, void* dS, void* dV, cudaStream_t cs, bool fpm = false) {
  std::lock_guard<std::mutex> lk(st->side_mu);
  return enqueue_full_locked(st, s, dO, P, Pd, V, M, p, dS, dV, cs, fpm);
}

// A full call as a CUDA graph: the first sighting of an argument list runs eagerly, the
// second captures the same launches (on a private stream, thread-local capture mode) into
// a graph, later ones replay it with one cudaGraphLaunch on the caller's stream, which
// removes most of the host-side launch cost for repeated calls on the same tensors.
// The replay depends only on the argument list (pointers, shape, dropout, stream): input
// contents may change freely between calls.  Option ATTN_BWD_OPT_GRAPH = 0 turns this off.
int run_full(DeviceState* st, const Shape& s, const void* dO, const void* P, const void* Pd, const void* V,
             const uint8_t* M, float p, void* dS, void* dV, cudaStream_t cs) {
  const bool graphs_on = opt(ATTN_BWD_OPT_GRAPH) != 0;
  if (!graphs_on) return enqueue_full(st, s, dO, P, Pd, V, M, p, dS, dV, cs);
  // a caller that is itself capturing this stream gets the plain launches in its graph
  cudaStreamCaptureStatus cap_status = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(cs, &cap_status) != cudaSuccess) return ATTN_BWD_ECUDA;
  if (cap_status != cudaStreamCaptureStatusNone) return enqueue_full(st, s, dO, P, Pd, V, M, p, dS, dV, cs);
  uint32_t pbits;
  std::memcpy(&pbits, &p, 4);
  // the options generation rides in the dropout word: a graph never outlives its options
  const uint64_t key[14] = {(uint64_t)dO, (uint64_t)P, (uint64_t)Pd, (uint64_t)V, (uint64_t)M, (uint64_t)dS,
                            (uint64_t)dV, pbits | ((uint64_t)g_opt_gen.load() << 32), (uint64_t)s.bs,
                            (uint64_t)s.sq, (uint64_t)s.skv, (uint64_t)s.u0, (uint64_t)s.u1, (uint64_t)cs};
  std::lock_guard<std::mutex> lk(st->side_mu);
  DeviceState::GraphEntry* hit = nullptr;
  DeviceState::GraphEntry* victim = &st->graphs[0];
  for (auto& g : st->graphs) {
    if (g.state && std::memcmp(g.key, key, sizeof(key)) == 0) { hit = &g; break; }
    if (!g.state || (victim->state && g.last_use < victim->last_use)) victim = &g;
  }
  const uint64_t now = ++st->graph_clock;
  if (hit && hit->state == 2) {
    hit->last_use = now;
    return cudaGraphLaunch(hit->exec, cs) == cudaSuccess ? ATTN_BWD_OK : ATTN_BWD_ECUDA;
  }
  if (!hit) {   // first sighting: remember it, run eagerly
    if (victim->state == 2) cudaGraphExecDestroy(victim->exec);
    std::memcpy(victim->key, key, sizeof(key));
    victim->state = 1;
    victim->last_use = now;
    victim->exec = nullptr;
    return enqueue_full_locked(st, s, dO, P, Pd, V, M, p, dS, dV, cs);
  }
  // second sighting: capture, instantiate, launch
  if (!st->cap && cudaStreamCreateWithFlags(&st->cap, cudaStreamNonBlocking) != cudaSuccess) return ATTN_BWD_ECUDA;
  cudaGraph_t graph = nullptr;
  if (cudaStreamBeginCapture(st->cap, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return ATTN_BWD_ECUDA;
  const int rc = enqueue_full_locked(st, s, dO, P, Pd, V, M, p, dS, dV, st->cap);
  const cudaError_t ce = cudaStreamEndCapture(st->cap, &graph);
  if (rc || ce != cudaSuccess || !graph) {
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    hit->state = 0;
    return rc ? rc : ATTN_BWD_ECUDA;
  }
  cudaGraphExec_t exec = nullptr;
  const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (ie != cudaSuccess) {
    hit->state = 0;
    return ATTN_BWD_ECUDA;
  }
  hit->exec = exec;
  hit->state = 2;
  hit->last_use = now;
  return cudaGraphLaunch(exec, cs) == cudaSuccess ? ATTN_BWD_OK : ATTN_BWD_ECUDA;
}


constexpr int kMaxHostChunks = 64;

// Units per alignment step of a shard boundary: the smallest g in {1,2,4,8} for which an
// offset of g units (10*g heads of sq*skv elements) is a multiple of 16 elements, so that
// every per-chunk slice of P / P_drop / mask / dS starts 16-byte aligned and keeps the row
// alignment classes of the whole call (the kernels then compute bit-identical rows).
int unit_step(int sq, int skv) {
  for (int g = 1; g < 8; g *= 2)
    if (((long long)kGroups * g * sq * skv) % 16 == 0) return g;
  return 8;
}

int make_host_resources(DeviceState* st) {
  if (st->h2d) return ATTN_BWD_OK;
  if (cudaStreamCreateWithFlags(&st->h2d, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&st->d2h, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&st->h_fork, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&st->h_join, cudaEventDisableTiming) != cudaSuccess)
    return ATTN_BWD_ECUDA;
  for (int k = 0; k < kMaxHostChunks; ++k)
    if (cudaEventCreateWithFlags(&st->in_done[k], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&st->comp_done[k], cudaEventDisableTiming) != cudaSuccess)
      return ATTN_BWD_ECUDA;
  return ATTN_BWD_OK;
}

inline bool copy_async(void* dst, const void* src, size_t bytes, cudaMemcpyKind kind, cudaStream_t s) {
  return bytes == 0 || cudaMemcpyAsync(dst, src, bytes, kind, s) == cudaSuccess;
}

// Host-buffer call as a three-stage pipeline over chunks of units:
//   stream h2d:  copy chunk k's inputs host -> device (dO rows of the batches it first
//                touches, its V slabs, its P / P_drop / mask heads), record in_done[k];
//   stream cs:   wait in_done[k], run the dS + dV kernels on chunk k (dV on the side
//                stream, joined back), record comp_done[k];
//   stream d2h:  wait comp_done[k], copy chunk k's dS heads and dV slabs device -> host.
// PCIe is full duplex and the copies of the two directions use separate copy engines, so
// the call takes about max(H2D bytes, D2H bytes) / PCIe bandwidth plus one chunk of
// latency, instead of the sum of both directions.  All three streams start after the work
// already on cs (fork event) and cs waits for the last device -> host copy (join event).
int run_host(DeviceState* st, const Shape& s, int chunks, const void* dO_h, const void* P_h, const void* Pd_h,
             const void* V_h, const uint8_t* M_h, float p, void* dS_h, void* dV_h, void* dO_d, void* P_d,
             void* Pd_d, void* V_d, uint8_t* M_d, void* dS_d, void* dV_d, cudaStream_t cs) {
  const int n_units = s.n_units();
  if (n_units == 0) return ATTN_BWD_OK;
  std::lock_guard<std::mutex> lk(st->host_mu);
  int rc = make_host_resources(st);
  if (rc) return rc;
  const int g = unit_step(s.sq, s.skv);
  // chunk boundaries are multiples of g units from unit_begin (which the caller's own
  // shard layout already aligns); a chunk never holds fewer than g units
  const int steps = (n_units + g - 1) / g;
  if (chunks <= 0) chunks = 16;
  if (chunks > kMaxHostChunks) chunks = kMaxHostChunks;
  if (chunks > steps) chunks = steps;
  const size_t head_elems = (size_t)s.sq * s.skv;                       // one head of P / mask / dS
  const size_t slab_elems = (size_t)s.skv * kHeadDim;                   // one unit of V / dV
  const size_t row_elems = (size_t)s.sq * kHeads * kHeadDim;            // one batch row of dO
  if (cudaEventRecord(st->h_fork, cs) != cudaSuccess || cudaStreamWaitEvent(st->h2d, st->h_fork, 0) != cudaSuccess ||
      cudaStreamWaitEvent(st->d2h, st->h_fork, 0) != cudaSuccess)
    return ATTN_BWD_ECUDA;
  int next_batch = 0;   // dO batch rows [0, next_batch) of the touched range are copied
  bool dO_any = false;
  for (int k = 0; k < chunks && rc == ATTN_BWD_OK; ++k) {
    // chunk k: units [a, b) relative to unit_begin, split as evenly as the step allows
    const int a = (int)((long long)steps * k / chunks) * g;
    int b = (int)((long long)steps * (k + 1) / chunks) * g;
    if (b > n_units) b = n_units;
    const int ua = s.u0 + a, ub = s.u0 + b;
    // ---- inputs
    const int b_lo = ua / kKvHeads, b_hi = (ub - 1) / kKvHeads + 1;   // batch rows this chunk reads
    int c_lo = dO_any && b_lo < next_batch ? next_batch : b_lo;
    bool ok = true;
    if (b_hi > c_lo) {
      const size_t off = (size_t)c_lo * row_elems * 2, bytes = (size_t)(b_hi - c_lo) * row_elems * 2;
      ok = copy_async((char*)dO_d + off, (const char*)dO_h + off, bytes, cudaMemcpyHostToDevice, st->h2d);
      next_batch = b_hi;
      dO_any = true;
    }
    const size_t h_off = (size_t)a * kGroups * head_elems, h_n = (size_t)(b - a) * kGroups * head_elems;
    const size_t v_off = (size_t)ua * slab_elems, v_n = (size_t)(b - a) * slab_elems;
    ok = ok && copy_async((char*)V_d + v_off * 2, (const char*)V_h + v_off * 2, v_n * 2, cudaMemcpyHostToDevice, st->h2d);
    ok = ok && copy_async((char*)P_d + h_off * 2, (const char*)P_h + h_off * 2, h_n * 2, cudaMemcpyHostToDevice, st->h2d);
    ok = ok && copy_async((char*)Pd_d + h_off * 2, (const char*)Pd_h + h_off * 2, h_n * 2, cudaMemcpyHostToDevice,
                          st->h2d);
    ok = ok && copy_async(M_d + h_off, M_h + h_off, h_n, cudaMemcpyHostToDevice, st->h2d);
    ok = ok && cudaEventRecord(st->in_done[k], st->h2d) == cudaSuccess;
    // ---- kernels
    ok = ok && cudaStreamWaitEvent(cs, st->in_done[k], 0) == cudaSuccess;
    if (!ok) { rc = ATTN_BWD_ECUDA; break; }
    const Shape cs_shape{s.bs, s.sq, s.skv, ua, ub};
    rc = enqueue_full(st, cs_shape, dO_d, (const char*)P_d + h_off * 2, (const char*)Pd_d + h_off * 2, V_d,
                      M_d + h_off, p, (char*)dS_d + h_off * 2, (char*)dV_d + (size_t)a * slab_elems * 2, cs);
    if (rc) break;
    // ---- outputs
    ok = cudaEventRecord(st->comp_done[k], cs) == cudaSuccess &&
         cudaStreamWaitEvent(st->d2h, st->comp_done[k], 0) == cudaSuccess &&
         copy_async((char*)dS_h + h_off * 2, (const char*)dS_d + h_off * 2, h_n * 2, cudaMemcpyDeviceToHost, st->d2h) &&
         copy_async((char*)dV_h + (size_t)a * slab_elems * 2, (const char*)dV_d + (size_t)a * slab_elems * 2,
                    v_n * 2, cudaMemcpyDeviceToHost, st->d2h);
    if (!ok) rc = ATTN_BWD_ECUDA;
  }
  // join even after an error, so cs never runs ahead of issued copies
  if (cudaEventRecord(st->h_join, st->h2d) != cudaSuccess || cudaStreamWaitEvent(cs, st->h_join, 0) != cudaSuccess ||
      cudaEventRecord(st->h_join, st->d2h) != cudaSuccess || cudaStreamWaitEvent(cs, st->h_join, 0) != cudaSuccess)
    return rc ? rc : ATTN_BWD_ECUDA;
  return rc;
}

}  // namespace

extern "C" {

int attn_bwd_b200_ds_shard(const void* dO, const void* P, const void* V, const uint8_t* M, float p, int bs, int sq,
                           int skv, int u0, int u1, void* dS, attn_bwd_stream_t stream) {
  Shape s{bs, sq, skv, u0, u1};
  DeviceState* st = nullptr;
  int rc = prologue(&st, s);
  if (rc) return rc;
  if (!ptr_ok(dO, s.n_dO()) || !ptr_ok(P, s.n_scores()) || !ptr_ok(V, s.n_V()) || !ptr_ok(M, s.n_scores()) ||
      !ptr_ok(dS, s.n_scores()))
    return ATTN_BWD_EINVAL;
  if (!aligned16(dO) || !aligned16(P) || !aligned16(V) || !aligned16(M) || !aligned16(dS)) return ATTN_BWD_EALIGN;
  return launch_ds(*st, s, dO, P, V, M, p, dS, reinterpret_cast<cudaStream_t>(stream));
}

int attn_bwd_b200_dv_shard(const void* dO, const void* Pd, int bs, int sq, int skv, int u0, int u1, void* dV,
                           attn_bwd_stream_t stream) {
  Shape s{bs, sq, skv, u0, u1};
  DeviceState* st = nullptr;
  int rc = prologue(&st, s);
  if (rc) return rc;
  if (!ptr_ok(dO, s.n_dO()) || !ptr_ok(Pd, s.n_scores()) || !ptr_ok(dV, s.n_dV())) return ATTN_BWD_EINVAL;
  if (!aligned16(dO) || !aligned16(Pd) || !aligned16(dV)) return ATTN_BWD_EALIGN;
  return launch_dv(*st, s, dO, Pd, dV, reinterpret_cast<cudaStream_t>(stream));
}

int attn_bwd_b200_shard(const void* dO, const void* P, const void* Pd, const void* V, const uint8_t* M, float p,
                        int bs, int sq, int skv, int u0, int u1, void* dS, void* dV, attn_bwd_stream_t stream) {
  Shape s{bs, sq, skv, u0, u1};
  DeviceState* st = nullptr;
  int rc = prologue(&st, s);
  if (rc) return rc;
  if (!ptr_ok(dO, s.n_dO()) || !ptr_ok(P, s.n_scores()) || !ptr_ok(Pd, s.n_scores()) || !ptr_ok(V, s.n_V()) ||
      !ptr_ok(M, s.n_scores()) || !ptr_ok(dS, s.n_scores()) || !ptr_ok(dV, s.n_dV()))
    return ATTN_BWD_EINVAL;
  if (!aligned16(dO) || !aligned16(P) || !aligned16(Pd) || !aligned16(V) || !aligned16(M) || !aligned16(dS) ||
      !aligned16(dV))
    return ATTN_BWD_EALIGN;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  return run_full(st, s, dO, P, Pd, V, M, p, dS, dV, cs);
}

int attn_bwd_b200_shard_from_mask(const void* dO, const void* P, const void* V, const uint8_t* M, float p, int bs,
                                  int sq, int skv, int u0, int u1, void* dS, void* dV, attn_bwd_stream_t stream) {
  if (!(p >= 0.f && p < 1.f)) return ATTN_BWD_EINVAL;
  Shape s{bs, sq, skv, u0, u1};
  DeviceState* st = nullptr;
  int rc = prologue(&st, s);
  if (rc) return rc;
  if (!ptr_ok(dO, s.n_dO()) || !ptr_ok(P, s.n_scores()) || !ptr_ok(V, s.n_V()) || !ptr_ok(M, s.n_scores()) ||
      !ptr_ok(dS, s.n_scores()) || !ptr_ok(dV, s.n_dV()))
    return ATTN_BWD_EINVAL;
  if (!aligned16(dO) || !aligned16(P) || !aligned16(V) || !aligned16(M) || !aligned16(dS) || !aligned16(dV))
    return ATTN_BWD_EALIGN;
  if (s.n_units() > 0 && s.sq > 0 && s.skv % 16) return ATTN_BWD_EUNSUPPORTED;
  return enqueue_full(st, s, dO, P, nullptr, V, M, p, dS, dV, reinterpret_cast<cudaStream_t>(stream), true);
}

int attn_bwd_b200(const void* dO, const void* P, const void* Pd, const void* V, const uint8_t* M, float p, int bs,
                  int sq, int skv, void* dS, void* dV, attn_bwd_stream_t stream) {
  return attn_bwd_b200_shard(dO, P, Pd, V, M, p, bs, sq, skv, 0, bs * kKvHeads, dS, dV, stream);
}

int attn_bwd_b200_host_shard(const void* dO_h, const void* P_h, const void* Pd_h, const void* V_h, const uint8_t* M_h,
                             float p, int bs, int sq, int skv, int u0, int u1, void* dS_h, void* dV_h, void* dO_d,
                             void* P_d, void* Pd_d, void* V_d, uint8_t* M_d, void* dS_d, void* dV_d, int chunks,
                             attn_bwd_stream_t stream) {
  Shape s{bs, sq, skv, u0, u1};
  DeviceState* st = nullptr;
  int rc = prologue(&st, s);
  if (rc) return rc;
  if (chunks < 0) return ATTN_BWD_EINVAL;
  const void* all[] = {dO_h, P_h, Pd_h, V_h, M_h, dS_h, dV_h, dO_d, P_d, Pd_d, V_d, M_d, dS_d, dV_d};
  const long long n[] = {s.n_dO(), s.n_scores(), s.n_scores(), s.n_V(), s.n_scores(), s.n_scores(), s.n_dV(),
                         s.n_dO(), s.n_scores(), s.n_scores(), s.n_V(), s.n_scores(), s.n_scores(), s.n_dV()};
  for (int i = 0; i < 14; ++i)
    if (!ptr_ok(all[i], n[i])) return ATTN_BWD_EINVAL;
  for (int i = 7; i < 14; ++i)
    if (!aligned16(all[i])) return ATTN_BWD_EALIGN;
  return run_host(st, s, chunks, dO_h, P_h, Pd_h, V_h, M_h, p, dS_h, dV_h, dO_d, P_d, Pd_d, V_d, M_d, dS_d, dV_d,
                  reinterpret_cast<cudaStream_t>(stream));
}

int attn_bwd_b200_host(const void* dO_h, const void* P_h, const void* Pd_h, const void* V_h, const uint8_t* M_h,
                       float p, int bs, int sq, int skv, void* dS_h, void* dV_h, void* dO_d, void* P_d, void* Pd_d,
                       void* V_d, uint8_t* M_d, void* dS_d, void* dV_d, int chunks, attn_bwd_stream_t stream) {
  return attn_bwd_b200_host_shard(dO_h, P_h, Pd_h, V_h, M_h, p, bs, sq, skv, 0, bs * kKvHeads, dS_h, dV_h, dO_d, P_d,
                                  Pd_d, V_d, M_d, dS_d, dV_d, chunks, stream);
}

int attn_bwd_b200_selftest_wait_timeout(int limit_us, attn_bwd_stream_t stream) {
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  if (limit_us <= 0 || limit_us > 1000000) return ATTN_BWD_EINVAL;
  wait_timeout_selftest<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      st->err, 0x7001, (unsigned long long)limit_us * 1000ull);
  return cudaPeekAtLastError() == cudaSuccess ? ATTN_BWD_OK : ATTN_BWD_ECUDA;
}

int attn_bwd_b200_poll_error(void) {
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  if (cudaDeviceSynchronize() != cudaSuccess) return ATTN_BWD_ECUDA;
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_kernel_error, sizeof(int)) != cudaSuccess) return ATTN_BWD_ECUDA;
  if (v && cudaMemcpyToSymbol(g_kernel_error, &zero, sizeof(int)) != cudaSuccess) return ATTN_BWD_ECUDA;
  return v;
}

const char* attn_bwd_b200_strerror(int code) {
  switch (code) {
    case ATTN_BWD_OK: return "ok";
    case ATTN_BWD_EINVAL: return "invalid argument (size, unit range or null pointer)";
    case ATTN_BWD_EALIGN: return "tensor pointer is not 16-byte aligned";
    case ATTN_BWD_EUNSUPPORTED: return "shape has no kernel path";
    case ATTN_BWD_ETMAP: return "TMA descriptor encoding failed";
    case ATTN_BWD_ECUDA: return "CUDA runtime call failed";
    case ATTN_BWD_EDEVICE: return "current device is not a compute capability 10.x (B200) GPU";
    case ATTN_BWD_EKERNEL: return "a kernel wait timed out";
    default: return "unknown error";
  }
}

int attn_bwd_b200_version(void) { return 102; }

int attn_bwd_b200_set_option(int option, int value) {
  if (option < 0 || option >= kNumOptions) return ATTN_BWD_EINVAL;
  g_opt[option].store(value);
  g_opt_gen.fetch_add(1);
  return ATTN_BWD_OK;
}

int attn_bwd_b200_get_option(int option) {
  if (option < 0 || option >= kNumOptions) return -2;
  return g_opt[option].load();
}

int attn_bwd_b200_release(void) {
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  if (cudaDeviceSynchronize() != cudaSuccess) return ATTN_BWD_ECUDA;
  std::lock_guard<std::mutex> lk_side(st->side_mu);
  std::lock_guard<std::mutex> lk_host(st->host_mu);
  bool ok = true;
  for (auto& g : st->graphs) {
    if (g.state == 2 && g.exec) ok &= cudaGraphExecDestroy(g.exec) == cudaSuccess;
    g = DeviceState::GraphEntry{};
  }
  auto drop_stream = [&](cudaStream_t& s) {
    if (s) ok &= cudaStreamDestroy(s) == cudaSuccess;
    s = nullptr;
  };
  auto drop_event = [&](cudaEvent_t& e) {
    if (e) ok &= cudaEventDestroy(e) == cudaSuccess;
    e = nullptr;
  };
  drop_stream(st->side);
  drop_stream(st->cap);
  drop_stream(st->h2d);
  drop_stream(st->d2h);
  drop_event(st->fork);
  drop_event(st->join);
  drop_event(st->h_fork);
  drop_event(st->h_join);
  for (int k = 0; k < kMaxHostChunks; ++k) {
    drop_event(st->in_done[k]);
    drop_event(st->comp_done[k]);
  }
  return ok ? ATTN_BWD_OK : ATTN_BWD_ECUDA;
}

#ifdef ATTN_BWD_WAIT_STATS
// Diagnostics builds only (not part of the ABI): copies and clears the per-site wait cycles.
int attn_bwd_b200_wait_stats(unsigned long long* out) {
  if (cudaDeviceSynchronize() != cudaSuccess) return ATTN_BWD_ECUDA;
  if (cudaMemcpyFromSymbol(out, sm100::g_wait_cycles, sizeof(unsigned long long) * 128) != cudaSuccess)
    return ATTN_BWD_ECUDA;
  static const unsigned long long zero[128] = {};
  return cudaMemcpyToSymbol(sm100::g_wait_cycles, zero, sizeof(zero)) == cudaSuccess ? ATTN_BWD_OK : ATTN_BWD_ECUDA;
}
#endif

}  // extern "C"
