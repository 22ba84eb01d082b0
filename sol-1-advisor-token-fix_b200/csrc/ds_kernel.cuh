// ds_kernel.cuh — fused dS kernel: dP~ = dO·Vᵀ on tcgen05 (TMEM accumulator),
// dropout backward and softmax backward in the epilogue, bf16 dS written once.
//
// Reference math (attn_bwd/starting_point.py:44-59, same as
// eval_modal_attn_bwd.py:108-124):
//   dP~ = dO_h · V_{h/10}ᵀ            (fp32)
//   dP  = dP~ · mask / (1 - p)        (only when p > 0)
//   r   = Σ_j dP_ij · P_ij
//   dS  = bf16(P · (dP − r))
//
// Work unit: one (batch·head, 128-row block of seq_q).  A unit is processed in
// 64-column chunks of seq_kv, twice: pass 1 accumulates the row sums r
// (thread-per-row, no shuffles), pass 2 forms dS.  The MMA for a chunk is
// re-issued in pass 2 (dP~ is never written to HBM) unless the whole row
// fits the TMEM ring with room for the next unit ("resident" mode, seq_kv <=
// 256), in which case pass 2 re-reads pass 1's TMEM columns.  P and the mask
// are streamed by TMA in both passes; pass 2 re-reads them from L2.
//
// Roles (640 threads):
//   warp 0  TMA producer for dO tiles and V chunks
//   warp 1  tcgen05 MMA issuer (also owns the TMEM allocation)
//   warp 2  P / mask producer
//   warp 3  dS store issuer (TMA tensor store of each finished chunk)
//   warps 4..19  epilogue; warp w reads TMEM lanes 32·(w%4).. and chunk
//                columns 16·((w-4)/4) ..+16
//
// Three row formats (template parameter RK):
//   kRowsAligned  seq_kv % 16 == 0: P / mask chunks are TMA tensor tiles
//                 (128B / 64B swizzle) and dS leaves by TMA tensor store.
//   kRowsRagged   any seq_kv: rows of P / mask are not 16-byte aligned, so each
//                 row segment is fetched by 16-byte cp.async from the 16-byte
//                 boundary below it into a padded row (pitch 144 B / 80 B); the
//                 epilogue re-aligns it in registers (funnel shifts), masks
//                 columns >= seq_kv, and stores dS through a per-warp transpose
//                 buffer with coalesced 2-byte stores.
//   kRowsClass    any seq_kv, rows grouped by alignment class.  Row R of the
//                 flat P buffer starts at element R·seq_kv, so its misalignment
//                 depends only on R mod 16, and rows 16 apart are 32·seq_kv
//                 bytes apart (a 16-byte multiple).  The 10 query heads of one
//                 (batch, kv-head) share V and are contiguous in P, so a unit is
//                 64 rows of class k plus 64 rows of class k+8 (k < 8) of one
//                 kv group: both share the P misalignment s = k·seq_kv mod 8.
//                 The MMA's V window is shifted to start at column -s, which
//                 makes every P / dS word of the tile 16-byte aligned: P and the
//                 mask arrive as per-class TMA boxes (2 each per chunk) in the
//                 aligned layouts, dO rows are gathered by cp.async, the
//                 epilogue is the aligned one (plus column bounds in the first
//                 and last chunk), and dS leaves by TMA store through a dS class
//                 map, except in a row's first and last chunk, where warp 3
//                 writes it with 16-byte stores.
#pragma once
#include "sm100.cuh"

namespace attn_bwd {

constexpr int kHeads = 80, kKvHeads = 8, kGroups = 10, kHeadDim = 128;

namespace ds {
constexpr int BM = 128;          // rows (seq_q) per unit
constexpr int BN = 64;           // columns (seq_kv) per chunk
constexpr int TSLOTS = 8;        // TMEM ring: 8 x 64 fp32 columns = 512
constexpr int RAG_P_PITCH = 144;   // ragged rows: 128 B of P row + 16 B of misalignment slack
constexpr int RAG_M_PITCH = 80;    // ragged rows: 64 B of mask row + 16 B of slack
constexpr int kEpiWarps = 16;                 // 4 per TMEM lane quadrant
constexpr int CW = BN / (kEpiWarps / 4);      // 16 chunk columns per epilogue thread
constexpr int kThreads = (4 + kEpiWarps) * 32;
constexpr int DO_BYTES = BM * kHeadDim * 2;   // 32 KB (two 64-column SW128 halves)
constexpr int V_BYTES = BN * kHeadDim * 2;    // 16 KB

// Pass-2 modes.
//   kRecompute  pass 2 re-issues the MMAs and re-reads P / mask (from L2); rows of any length.
//   kResident   dP~ stays in TMEM (8 slots of 64 columns), pass 2 re-reads P / mask from L2.
//   kTmemP      pass 1 writes the masked dP~ (fp32) and P (bf16 pairs) back into TMEM
//               (96-column slots, <= 5 chunks per CTA), so pass 2 reads TMEM only and the
//               whole shared-memory ring prefetches pass-1 data from HBM.
//   kCompact    MMAs land in a ring of 3 fp32 slots; pass 1 writes the masked dP~ back as
//               bf16 pairs (32 columns per chunk) and frees the slot at once, so one CTA
//               holds rows of up to 10 chunks (640 columns) without a cluster.  Pass 2
//               re-reads P from L2.  Rounding dP~ to bf16 adds at most ~|P|·|dP~|·2^-9 to dS.
enum Mode : int { kRecompute = 0, kResident = 1, kTmemP = 2, kCompact = 3 };
enum RowKind : int { kRowsAligned = 0, kRowsRagged = 1, kRowsClass = 2 };
constexpr int CLS_M_PITCH = 80;   // class rows: 64 B of mask row + 16 B (window may start 8 B into a word)

// Stage counts of the aligned kCompact form (compile-time tuning overrides for measurements).
#ifndef ATTN_BWD_RES_VST
#define ATTN_BWD_RES_VST 2
#endif
#ifndef ATTN_BWD_RES_PST
#define ATTN_BWD_RES_PST 6
#endif
// class-tile rows with dP~ resident: a third V stage fits beside the five P / mask stages and
// lets the MMA run further ahead of the epilogue (c2 dS 237.5 -> 227.4 us, 8x373x449 204.8 ->
// 198.8 us).  Aligned resident rows keep 2 V + 6 P / mask stages (3 + 5 measured +2 % on c1,
// -3 % on c3's clusters).
#ifndef ATTN_BWD_CLS_VST
#define ATTN_BWD_CLS_VST 3
#endif
#ifndef ATTN_BWD_CP_VST
#define ATTN_BWD_CP_VST 2
#endif
#ifndef ATTN_BWD_CP_PST
#define ATTN_BWD_CP_PST 6
#endif

// Shared-memory plan per mode.  With dP~ resident the MMAs of a unit end with
// pass 1, so one dO buffer suffices and the freed space buys P/mask stages
// (bytes in flight are what keep HBM busy).
template <int RK, int MODE>
struct Cfg {
  static constexpr bool RAG = RK == kRowsRagged;
  static constexpr bool CLS = RK == kRowsClass;
  static constexpr bool RES = MODE != kRecompute;     // each chunk's MMA is issued once
  static constexpr bool HOLD = MODE == kResident || MODE == kTmemP;   // slots held until pass 2
  static constexpr bool CP = MODE == kCompact;
  static constexpr int CP_SLOTS = 3;                   // kCompact: fp32 ring slots
  static constexpr int CP_BASE = CP_SLOTS * BN;        // kCompact: first column of the bf16 store
  static constexpr int CP_MAX = (TSLOTS * BN - CP_BASE) / (BN / 2);   // kCompact: chunks per CTA (10)
  static constexpr bool TP = MODE == kTmemP;
  static constexpr int DOBUF = RES ? 1 : 2;            // dO tile buffers
  // V chunk stages (aligned non-resident: V read twice); P/mask chunk stages
  static constexpr bool ALRES = RK == kRowsAligned && MODE == kResident;
  static constexpr bool CLSRES = CLS && MODE == kResident;
  static constexpr int VST = (CP && !CLS) ? ATTN_BWD_CP_VST : ALRES ? ATTN_BWD_RES_VST : CLSRES ? ATTN_BWD_CLS_VST
                           : RAG ? 2 : RES ? 2 : 3;
  static constexpr int PST = (CP && !CLS) ? ATTN_BWD_CP_PST : ALRES ? ATTN_BWD_RES_PST : TP ? 4 : RAG ? (RES ? 4 : 3)
                           : CLS ? (RES ? 5 : 3) : (RES ? 6 : 4);
  static constexpr int SLOTC = TP ? 96 : BN;           // TMEM columns per chunk slot
  static constexpr int NSLOT = TP ? 5 : CP ? CP_SLOTS : TSLOTS;   // TMEM slots (<= 512 columns)
  static constexpr int DST_BYTES = (TP && !RAG) ? 2 * BM * BN * 2 : 0;   // dS staging tiles (SW128)
  static constexpr int P_PITCH = RAG ? RAG_P_PITCH : 128;  // bytes per staged P row
  static constexpr int M_PITCH = RAG ? RAG_M_PITCH : CLS ? CLS_M_PITCH : 64;   // bytes per staged mask row
  static constexpr int P_BYTES = BM * P_PITCH;
  static constexpr int M_BYTES = BM * M_PITCH;
  static constexpr int STG_PITCH = 48;                 // per-warp dS transpose rows (RAG): 32 B + pad
  static constexpr int STG_BYTES = RAG ? kEpiWarps * 32 * STG_PITCH : 0;
  static constexpr int OFF_DO = 0;
  static constexpr int OFF_V = OFF_DO + DOBUF * DO_BYTES;
  static constexpr int OFF_P = OFF_V + VST * V_BYTES;
  static constexpr int OFF_M = OFF_P + PST * P_BYTES;
  static constexpr int OFF_STG = OFF_M + PST * M_BYTES;
  static constexpr int OFF_DST = OFF_STG + STG_BYTES;
  static constexpr int OFF_BAR = OFF_DST + DST_BYTES;
  // barriers: dO full/empty (2+2), V full/empty, PM full/empty, dS ready, T full/empty, quad (4)
  static constexpr int NBAR = 4 + 2 * VST + 3 * PST + 2 * TSLOTS + 4 + 2;
  static_assert(DOBUF <= 2, "two dO barrier slots");
  static constexpr int OFF_RX = OFF_BAR + NBAR * 8;    // float rx[2][4][128]: per-column-group row sums
  static constexpr int OFF_XB = OFF_RX + 2 * 4 * BM * 4;   // float xb[2][8][128]: row sums from each cluster CTA
  static constexpr int OFF_MISC = OFF_XB + 2 * 8 * BM * 4;   // tmem base, abort flag, cluster exchange barrier
  static constexpr int OFF_DOTAB = OFF_MISC + 64;             // class rows: byte offsets of the tile's 128 dO rows
  static constexpr int SMEM_BYTES = OFF_DOTAB + (CLS ? BM * 8 : 0) + 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "dS kernel shared memory");
};

struct Params {
  int sq, skv;
  int n_units;      // local (batch·head) count × row blocks
  int n_mb;         // row blocks per head
  int nchunks;      // ceil(skv / 64)
  int cs;           // CTAs per cluster sharing one unit's columns (1: no cluster)
  int cpc;          // chunks per CTA of a cluster (CTA k owns chunks [k·cpc, (k+1)·cpc))
  int resident;     // 1: pass 2 re-reads pass-1 TMEM columns
  int bh_base;      // global (batch·head) index of local head 0
  int use_mask;     // p > 0
  int l2pf;         // aligned rows, two passes: L2 prefetch of the next unit during pass 2
  int l2hint;       // aligned rows: L2 eviction hints (pass-1 tiles kept, pass-2 tiles and dS evicted first)
  float scale;      // 1/(1-p) when use_mask, else 1
  int* err;
  // raw pointers for the RAG path (local shard bases, 16-byte aligned)
  const uint8_t* P;
  const uint8_t* M;
  uint8_t* dS;
  unsigned long long p_end16;   // bytes of P rounded up to 16 (bulk copies never read past it)
  unsigned long long m_end16;   // same for the mask
  // kRowsClass
  const uint8_t* dO;            // dO base ([bs, sq, 80, 128]); rows are gathered by cp.async
  int cls_T;                    // 64-row tiles per class per kv group
  int cls_Y;                    // 16-row groups of the local P buffer the class tensor maps cover
};

// kRowsClass unit u = (local kv group ul, tile t, class pair k), k fastest.
struct ClsUnit {
  long long g0;     // local flat row of the group's first row (ul · 10 · sq)
  int rho[2];       // group row of tile row 0 of sub-class A (class k) / B (class k+8); rows step 16
  int cls[2];       // the two classes (R mod 16)
  int s;            // P misalignment of the tile's rows in elements: chunk c covers columns 64c-s ..
  int mo[2];        // byte offset (0 or 8) of each sub-class's mask window inside its 16-byte word
  int zv;           // V index b·8 + kv-head
  int ug;           // global (batch, kv-head) index
  bool fallback;    // a row lies past the class maps' extent: fetch by cp.async
  bool pad;         // a sub-class has fewer than 64 rows: the tile holds padding rows
};

__device__ __forceinline__ ClsUnit cls_unit(int u, const Params& prm) {
  ClsUnit x;
  const int T = prm.cls_T;
  // the 8 class pairs of one row range are consecutive units, so neighbouring CTAs read
  // the 16 classes of the same 16-row groups at the same time (DRAM page locality)
  const int k = u & 7;
  const int t = (u >> 3) % T;
  const int ul = u / (8 * T);
  const int rows = kGroups * prm.sq;
  x.g0 = (long long)ul * rows;
  x.s = (k * prm.skv) & 7;
  x.fallback = false;
  x.pad = false;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int cl = k + 8 * h;
    x.cls[h] = cl;
    const int r0 = int(((long long)cl - x.g0) & 15);   // first group row of this class
    const int n = r0 < rows ? (rows - 1 - r0) / 16 + 1 : 0;   // rows of this class in the group
    // tile t covers class rows [64t, 64t+64); the last tile is moved back to end at row n,
    // overlapping its predecessor (rows computed twice get bit-identical values), so only
    // classes with fewer than 64 rows leave padding rows in a tile
    const int b0 = min(64 * t, max(n - 64, 0));
    if (n < 64) x.pad = true;
    x.rho[h] = r0 + 16 * b0;
    x.mo[h] = int(((long long)cl * prm.skv - x.s) & 15);
    if (x.rho[h] < rows) {
      const int last = min(x.rho[h] + 16 * 63, x.rho[h] + 16 * ((rows - 1 - x.rho[h]) / 16));
      if ((x.g0 + last) / 16 >= prm.cls_Y) x.fallback = true;
    }
  }
  x.ug = prm.bh_base / kGroups + ul;
  x.zv = x.ug;
  return x;
}

// Shifts a little-endian byte stream right by `sh` bytes (0..15):
// out[j] = bytes [4j+sh, 4j+sh+4) of `in`.  `in` holds NOUT+4 words.
template <int NOUT>
__device__ __forceinline__ void byte_shift(const uint32_t* in, uint32_t sh, uint32_t* out) {
  uint32_t u[NOUT + 2], v[NOUT + 1];
#pragma unroll
  for (int j = 0; j < NOUT + 2; ++j) u[j] = (sh & 8) ? in[j + 2] : in[j];
#pragma unroll
  for (int j = 0; j < NOUT + 1; ++j) v[j] = (sh & 4) ? u[j + 1] : u[j];
  const uint32_t bits = (sh & 3) * 8;
#pragma unroll
  for (int j = 0; j < NOUT; ++j) out[j] = __funnelshift_r(v[j], v[j + 1], bits);
}

// Loads this thread's 16 P values (8 words of bf16 pairs) and 16 mask bytes
// (4 words) of one chunk row, column group `cg` (columns 16·cg .. +16).
template <bool RAG>
__device__ __forceinline__ void load_row(uint32_t p_stage, uint32_t m_stage, int row, int cg, uint32_t shP,
                                         uint32_t shM, uint32_t (&pw)[8], uint32_t (&mw)[4]) {
  using namespace sm100;
  if constexpr (!RAG) {
    // TMA 128B swizzle: 16-byte chunk j of row r sits at chunk j ^ (r % 8); 64B swizzle: j ^ ((r/2) % 4)
    const uint32_t p_row = p_stage + row * 128;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint4 t = lds128(p_row + (((cg * 2 + i) ^ (row & 7)) << 4));
      pw[4 * i] = t.x; pw[4 * i + 1] = t.y; pw[4 * i + 2] = t.z; pw[4 * i + 3] = t.w;
    }
    const uint4 t = lds128(m_stage + row * 64 + ((cg ^ ((row >> 1) & 3)) << 4));
    mw[0] = t.x; mw[1] = t.y; mw[2] = t.z; mw[3] = t.w;
  } else {
    uint32_t in[12];
    const uint32_t p_row = p_stage + row * RAG_P_PITCH + cg * 32;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const uint4 t = lds128(p_row + i * 16);
      in[4 * i] = t.x; in[4 * i + 1] = t.y; in[4 * i + 2] = t.z; in[4 * i + 3] = t.w;
    }
    byte_shift<8>(in, shP, pw);
    const uint32_t m_row = m_stage + row * RAG_M_PITCH + cg * 16;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint4 t = lds128(m_row + i * 16);
      in[4 * i] = t.x; in[4 * i + 1] = t.y; in[4 * i + 2] = t.z; in[4 * i + 3] = t.w;
    }
    byte_shift<4>(in, shM, mw);
  }
}

// Keep-masks for 16 elements: mx[i] holds 4 bytes 0x00 / 0xFF (mask bytes are
// bool 0/1, so ×0xFF never carries); element e's 32-bit mask is byte e%4 of
// mx[e/4] replicated.  All-ones when the mask is not applied (p <= 0).
__device__ __forceinline__ void expand_mask(const uint32_t (&mw)[4], int use_mask, uint32_t (&mx)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) mx[i] = use_mask ? mw[i] * 0xFFu : 0xFFFFFFFFu;
}
__device__ __forceinline__ uint32_t mask_at(const uint32_t (&mx)[4], int e) {
  return __byte_perm(mx[e >> 2], 0u, (e & 3) * 0x1111u);
}

// kRowsClass: P as in the aligned layout (128B swizzle); mask rows at pitch 80 with the
// window starting `mo` (0 or 8, uniform per warp) bytes into the row.
__device__ __forceinline__ void load_row_cls(uint32_t p_stage, uint32_t m_stage, int row, int cg, int mo,
                                             uint32_t (&pw)[8], uint32_t (&mw)[4]) {
  using namespace sm100;
  const uint32_t p_row = p_stage + row * 128;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint4 t = lds128(p_row + (((cg * 2 + i) ^ (row & 7)) << 4));
    pw[4 * i] = t.x; pw[4 * i + 1] = t.y; pw[4 * i + 2] = t.z; pw[4 * i + 3] = t.w;
  }
  const uint32_t m_addr = m_stage + row * CLS_M_PITCH + cg * 16;
  if (mo == 0) {
    const uint4 t = lds128(m_addr);
    mw[0] = t.x; mw[1] = t.y; mw[2] = t.z; mw[3] = t.w;
  } else {
    uint32_t a, b, c2, d;
    asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];" : "=r"(a), "=r"(b) : "r"(m_addr + 8));
    asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];" : "=r"(c2), "=r"(d) : "r"(m_addr + 16));
    mw[0] = a; mw[1] = b; mw[2] = c2; mw[3] = d;
  }
}

// Ragged rows: dS of this warp's 32 rows x 16 columns goes out through the
// warp's transpose buffer, so each 2-byte store instruction writes 2 rows x 32
// contiguous bytes instead of 32 scattered rows.
template <int STG_PITCH>
__device__ __forceinline__ void store_rag_dS_impl(const uint32_t (&o)[8], uint32_t stg, uint32_t lane, const Params& prm,
                                                  int bhl, int sq, int skv, int mb, int q, int c, int cg) {
  using namespace sm100;
  const uint32_t srow = stg + lane * STG_PITCH;
  sts128(srow, make_uint4(o[0], o[1], o[2], o[3]));
  sts128(srow + 16, make_uint4(o[4], o[5], o[6], o[7]));
  __syncwarp();
  const int col = c * BN + cg * CW + int(lane & 15);
  const int rows_here = min(32, sq - (mb * BM + q * 32));
  if (col < skv) {
    unsigned short* dst =
        reinterpret_cast<unsigned short*>(prm.dS) + ((unsigned long long)bhl * sq + mb * BM + q * 32) * skv + col;
    for (int rr = int(lane >> 4); rr < rows_here; rr += 2) {
      unsigned short val;
      asm volatile("ld.shared.u16 %0, [%1];" : "=h"(val) : "r"(stg + rr * STG_PITCH + (lane & 15) * 2));
      dst[(unsigned long long)rr * skv] = val;
    }
  }
  __syncwarp();
}
#define store_rag_dS(o, stg, lane, prm, bhl, sq, skv, mb, q, c, cg) \
  store_rag_dS_impl<C::STG_PITCH>(o, stg, lane, prm, bhl, sq, skv, mb, q, c, cg)

// kRowsClass: a chunk goes out by TMA store (one 64 x 64 box per sub-class through the dS
// class map) when every word of it belongs to the tile's rows: no padding rows, rows inside
// the map, and the 64-column window inside the row.
__device__ __forceinline__ bool cls_tma_store_ok(const ClsUnit& cu, int c, const Params& prm) {
  const int col = c * BN - cu.s;
  return !cu.pad && !cu.fallback && col >= 0 && col + BN <= prm.skv;
}
__device__ __forceinline__ bool cls_tma_unit_ok(bool unit_ok, int c, int s, int skv) {
  const int col = c * BN - s;
  return unit_ok && col >= 0 && col + BN <= skv;
}
__device__ __forceinline__ void cls_tma_store(const CUtensorMap* tm, uint8_t* tile, const ClsUnit& cu, int c, int skv,
                                              bool hint = false) {
  const int col = c * BN - cu.s;
  const uint64_t pol = hint ? sm100::policy_evict_first() : 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int x = (h ? cu.cls[1] : cu.cls[0]) * skv + col, y = int((cu.g0 + (h ? cu.rho[1] : cu.rho[0])) >> 4);
    if (hint)
      sm100::tma_store_2d_hint(tm, tile + h * (BM * BN), x, y, pol);
    else
      sm100::tma_store_2d(tm, tile + h * (BM * BN), x, y);
  }
}

// kRowsClass: writes one finished 128 x 64 dS chunk from a 128B-swizzled staging tile.
// Lane = (row lane/8 of 4, 16-byte word lane%8): 4 rows x 128 B per store instruction.
// Every word is 16-byte aligned (the window starts at column -s); words that straddle a
// row end (first chunk when s > 0, last chunk) go out element by element, and padding
// rows (past the kv group) are skipped.
__device__ __forceinline__ void cls_store_chunk(uint32_t tile, const ClsUnit& cu, int c, const Params& prm,
                                                uint32_t lane) {
  using namespace sm100;
  const int rows = kGroups * prm.sq, skv = prm.skv;
  const int j = int(lane & 7);
  const int col = c * BN - cu.s + 8 * j;
  if (col + 8 <= 0 || col >= skv) return;
  const bool full = col >= 0 && col + 8 <= skv;
#pragma unroll 4
  for (int it = 0; it < BM / 4; ++it) {
    const int i = 4 * it + int(lane >> 3);
    const int rho = (i < 64 ? cu.rho[0] : cu.rho[1]) + 16 * (i & 63);
    if (rho < rows) {
      const uint4 v = lds128(tile + i * 128 + ((j ^ (i & 7)) << 4));
      uint8_t* dst = prm.dS + 2 * ((unsigned long long)(cu.g0 + rho) * skv + col);
      if (full) {
        *reinterpret_cast<uint4*>(dst) = v;
      } else {
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (col + e >= 0 && col + e < skv)
            reinterpret_cast<unsigned short*>(dst)[e] = (unsigned short)(wv[e >> 1] >> ((e & 1) * 16));
      }
    }
  }
}

template <int RK, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
ds_kernel(const __grid_constant__ CUtensorMap tm_dO,   // (d, h, s, b)   box (64,1,128,1) SW128
          const __grid_constant__ CUtensorMap tm_V,    // (d, skv, b·8)  box (64,64,1)    SW128
          const __grid_constant__ CUtensorMap tm_P,    // aligned: (skv, sq, bh) box (64,128,1) SW128;
                                                       // class: (16·skv, rows/16) box (64,64) SW128
          const __grid_constant__ CUtensorMap tm_M,    // aligned: (skv, sq, bh) box (64,128,1) SW64 u8;
                                                       // class: u8 (16·skv, rows/16) box (80,64)
          const __grid_constant__ CUtensorMap tm_dS,   // aligned: (skv, sq, bh) box (64,128,1) SW128;
                                                       // class: as tm_P
          const Params prm) {
  using namespace sm100;
  using C = Cfg<RK, MODE>;
  constexpr bool RAG = C::RAG, CLS = C::CLS;
  constexpr int PST = C::PST, VST = C::VST, DOBUF = C::DOBUF;
  constexpr bool RES = C::RES, TP = C::TP, HOLD = C::HOLD, CP = C::CP;
  constexpr int NSLOT = C::NSLOT, SLOTC = C::SLOTC;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* dO_full = bars + 0;
  uint64_t* dO_empty = bars + 2;
  uint64_t* V_full = bars + 4;
  uint64_t* V_empty = V_full + VST;
  uint64_t* PM_full = V_empty + VST;
  uint64_t* PM_empty = PM_full + PST;
  uint64_t* dS_ready = PM_empty + PST;
  uint64_t* T_full = dS_ready + PST;
  uint64_t* T_empty = T_full + TSLOTS;
  uint64_t* pair_bar = T_empty + TSLOTS;
  uint64_t* dS_free = pair_bar + 4;   // kTmemP: dS staging tile free again (store has read it)
  float* rx = reinterpret_cast<float*>(smem + C::OFF_RX);
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  uint64_t* xbar = reinterpret_cast<uint64_t*>(smem + C::OFF_MISC + 16);
  float* xb = reinterpret_cast<float*>(smem + C::OFF_XB);

  ATTN_BWD_WAIT_STATS_BEGIN();
  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    for (int i = 0; i < DOBUF; ++i) { mbar_init(&dO_full[i], CLS ? 32 : 1); mbar_init(&dO_empty[i], 1); }
    for (int i = 0; i < VST; ++i) { mbar_init(&V_full[i], 1); mbar_init(&V_empty[i], 1); }
    for (int i = 0; i < PST; ++i) {
      mbar_init(&PM_full[i], RAG ? 64 : 1);   // RAG: one cp.async completion arrive per producer lane (2 warps)
      mbar_init(&PM_empty[i], kEpiWarps);
      mbar_init(&dS_ready[i], kEpiWarps);
    }
    for (int i = 0; i < TSLOTS; ++i) { mbar_init(&T_full[i], 1); mbar_init(&T_empty[i], kEpiWarps); }
    for (int i = 0; i < 4; ++i) mbar_init(&pair_bar[i], 32 * (kEpiWarps / 4));
    for (int i = 0; i < 2; ++i) mbar_init(&dS_free[i], 1);
    // every CTA of the cluster (itself included) arrives once per row per unit
    mbar_init(xbar, prm.cs * BM);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_V);
    if (!CLS) prefetch_tmap(&tm_dO);
    if (!RAG && !CLS) { prefetch_tmap(&tm_P); prefetch_tmap(&tm_M); prefetch_tmap(&tm_dS); }
    if (CLS && prm.cls_Y > 0) { prefetch_tmap(&tm_P); prefetch_tmap(&tm_M); prefetch_tmap(&tm_dS); }
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_slot, TSLOTS * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  if (prm.cs > 1) cluster_sync();   // peers' barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  const int n_units = prm.n_units, n_mb = prm.n_mb, nchunks = prm.nchunks;
  // Cluster split of long rows: the cs CTAs of a cluster process the same units,
  // CTA `rank` owning chunks [c0, c0 + nloc) of every row; persistent over units
  // by cluster.  cs == 1: plain launch, one CTA owns whole rows.
  const int cs = prm.cs;
  const int rank = cs > 1 ? int(cluster_ctarank()) : 0;
  const int cid = int(blockIdx.x) / cs, ncl = int(gridDim.x) / cs;
  const int c0 = rank * prm.cpc;
  const int nloc = max(0, min(prm.cpc, nchunks - c0));
  const int sq = prm.sq, skv = prm.skv;
  constexpr int npass_mma = RES ? 1 : 2;
  int* err = prm.err;

  if (warp == 0) {
    // ------------------------------------------------ dO / V producer (lane 0 issues)
    uint32_t vi = 0, di = 0;
    for (int u = cid; u < n_units; u += ncl) {
      int zv, vshift = 0;
      const int db = di % DOBUF;
      if (!warp_wait(&dO_empty[db], ((di / DOBUF) & 1) ^ 1, abort_flag, err, 0x0101)) goto producer_done;
      if constexpr (CLS) {
        // gather the tile's 128 dO rows (sub-class A rows 0..63, B rows 64..127) by 16-byte
        // cp.async into the 128B-swizzled K-major layout a TMA box would produce
        const ClsUnit cu = cls_unit(u, prm);
        zv = cu.zv;
        vshift = cu.s;
        const int b = cu.ug / kKvHeads, kvh = cu.ug - b * kKvHeads;
        const int rows = kGroups * sq;
        // byte offsets of the 128 dO rows into a table (read back by this warp before each
        // copy is issued, so the next unit may overwrite it)
        unsigned long long* tab = reinterpret_cast<unsigned long long*>(smem + C::OFF_DOTAB);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int i = int(lane) + 32 * m;
          int rho = (i < 64 ? cu.rho[0] : cu.rho[1]) + 16 * (i & 63);
          if (rho >= rows) rho = cu.rho[0] < rows ? cu.rho[0] : 0;   // padding row: any valid row
          const int hl = rho / sq, sqi = rho - hl * sq;
          tab[i] = (((unsigned long long)b * sq + sqi) * kHeads + kvh * kGroups + hl) * (kHeadDim * 2);
        }
        __syncwarp();
        const uint32_t base = smem_u32(smem + C::OFF_DO + db * DO_BYTES);
        const int w = int(lane & 15), hf = w >> 3, j = w & 7;
#pragma unroll 4
        for (int it = 0; it < 64; ++it) {
          const int i = 2 * it + int(lane >> 4);   // 16 lanes per row: 2 rows x 256 B per step
          cp_async16(base + hf * (DO_BYTES / 2) + i * 128 + ((j ^ (i & 7)) << 4), prm.dO + tab[i] + w * 16);
        }
        // each lane's copies complete into dO_full (count 32); the MMA warp orders them
        // before its tensor-core reads with a proxy fence
        cp_async_arrive_noinc(&dO_full[db]);
        __syncwarp();
      } else {
        const int bhl = u / n_mb, mb = u - bhl * n_mb;
        const int bh = prm.bh_base + bhl;
        const int b = bh / kHeads, h = bh - b * kHeads;
        zv = b * kKvHeads + h / kGroups;
        if (lane == 0) {
          mbar_arrive_expect_tx(&dO_full[db], DO_BYTES);
          tma_load_4d(smem + C::OFF_DO + db * DO_BYTES, &tm_dO, &dO_full[db], 0, h, mb * BM, b);
          tma_load_4d(smem + C::OFF_DO + db * DO_BYTES + DO_BYTES / 2, &tm_dO, &dO_full[db], 64, h, mb * BM, b);
        }
      }
      ++di;
      for (int pass = 0; pass < npass_mma; ++pass) {
        for (int cl = 0; cl < nloc; ++cl) {
          const int c = c0 + cl;
          const int vs = vi % VST;
          if (!warp_wait(&V_empty[vs], ((vi / VST) & 1) ^ 1, abort_flag, err, 0x0102)) goto producer_done;
          if (lane == 0) {
            mbar_arrive_expect_tx(&V_full[vs], V_BYTES);
            uint8_t* dst = smem + C::OFF_V + vs * V_BYTES;
            // class rows: the window starts at column -s (V rows below 0 read as zeros)
            tma_load_3d(dst, &tm_V, &V_full[vs], 0, c * BN - vshift, zv);
            tma_load_3d(dst + V_BYTES / 2, &tm_V, &V_full[vs], 64, c * BN - vshift, zv);
          }
          ++vi;
        }
      }
    }
  producer_done:
    if (CLS) cp_async_wait_all();
    // drain: the last issue of every stage must have landed before exit
    if (lane == 0) {
      for (uint32_t k = 0; k < uint32_t(DOBUF) && k < di; ++k) {
        const uint32_t i = di - 1 - k;
        mbar_drain(&dO_full[i % DOBUF], (i / DOBUF) & 1, err, 0x0111);
      }
      for (uint32_t k = 0; k < uint32_t(VST) && k < vi; ++k) {
        const uint32_t i = vi - 1 - k;
        mbar_drain(&V_full[i % VST], (i / VST) & 1, err, 0x0112);
      }
    }
    __syncwarp();
  } else if (warp == 2 || (RAG && warp == 3)) {
    // ------------------------------------------------ P / mask producer (RAG: warps 2 and 3)
    uint32_t pi = 0;
    for (int u = cid; u < n_units; u += ncl) {
      const int bhl = CLS ? 0 : u / n_mb, mb = CLS ? 0 : u - bhl * n_mb;
      ClsUnit cu;
      if constexpr (CLS) cu = cls_unit(u, prm);
      for (int pass = 0; pass < (TP ? 1 : 2); ++pass) {
        for (int cl = 0; cl < nloc; ++cl) {
          const int c = c0 + cl;
          const int ps = pi % PST;
          if (!warp_wait(&PM_empty[ps], ((pi / PST) & 1) ^ 1, abort_flag, err, 0x0103)) goto pm_done;
          if constexpr (CLS) {
            uint8_t* pdst = smem + C::OFF_P + ps * C::P_BYTES;
            uint8_t* mdst = smem + C::OFF_M + ps * C::M_BYTES;
            const int col0 = c * BN - cu.s;   // window start column (a multiple of 8 elements from the row start's class offset)
            if (!cu.fallback) {
              // per sub-class: one P box (64 rows x 128 B, SW128) and one mask box (64 rows x 80 B)
              const bool want_m = !(CP && pass == 1);   // kCompact's pass 2 needs P alone
              if (lane == 0) mbar_arrive_expect_tx(&PM_full[ps], C::P_BYTES + (want_m ? C::M_BYTES : 0));
              __syncwarp();
              if (lane < (want_m ? 4 : 2)) {
                const int h = lane & 1;
                const int y = int((cu.g0 + (h ? cu.rho[1] : cu.rho[0])) >> 4);
                const int xe = (h ? cu.cls[1] : cu.cls[0]) * skv + col0;   // element offset inside the 16-row group
                if (prm.l2hint) {
                  // as on the aligned path: pass-1 tiles kept for pass 2, pass-2 reloads evicted first
                  const uint64_t pol = (pass == 0 && !TP) ? policy_evict_last() : policy_evict_first();
                  if (lane < 2)
                    tma_load_2d_hint(pdst + h * (C::P_BYTES / 2), &tm_P, &PM_full[ps], xe, y, pol);
                  else
                    tma_load_2d_hint(mdst + h * (C::M_BYTES / 2), &tm_M, &PM_full[ps], xe - (h ? cu.mo[1] : cu.mo[0]),
                                     y, pol);
                } else if (lane < 2) {
                  tma_load_2d(pdst + h * (C::P_BYTES / 2), &tm_P, &PM_full[ps], xe, y);
                } else {
                  tma_load_2d(mdst + h * (C::M_BYTES / 2), &tm_M, &PM_full[ps], xe - (h ? cu.mo[1] : cu.mo[0]), y);
                }
              }
            } else {
              // rows past the class maps' extent: 16-byte cp.async per row into the same layouts
              // (P: 8 words, 128B swizzle; mask: 5 words at pitch 80), then complete at once
              const uint32_t ps_u = smem_u32(pdst), ms_u = smem_u32(mdst);
              const int w = int(lane & 15);
              const int rows = kGroups * sq;
              for (int it = 0; it < BM / 2; ++it) {
                const int i = 2 * it + int(lane >> 4);
                const int h = i >> 6;
                const int rho = (h ? cu.rho[1] : cu.rho[0]) + 16 * (i & 63);
                if (rho >= rows) continue;
                const long long R = cu.g0 + rho;
                if (w < 8) {
                  const unsigned long long sp = (unsigned long long)(R * skv + col0) * 2 + 16ull * w;
                  if (sp < prm.p_end16) cp_async16(ps_u + i * 128 + ((w ^ (i & 7)) << 4), prm.P + sp);
                } else if (w < 13) {
                  const unsigned long long sm_ = (unsigned long long)(R * skv + col0 - (h ? cu.mo[1] : cu.mo[0])) + 16ull * (w - 8);
                  if (sm_ < prm.m_end16) cp_async16(ms_u + i * CLS_M_PITCH + (w - 8) * 16, prm.M + sm_);
                }
              }
              cp_async_wait_all();
              __syncwarp();
              if (lane == 0) mbar_arrive(&PM_full[ps]);
            }
          } else if constexpr (!RAG) {
            if (lane == 0) {
              // kCompact keeps the MASKED dP~, so its pass 2 needs P alone
              const bool want_m = !(CP && pass == 1);
              mbar_arrive_expect_tx(&PM_full[ps], C::P_BYTES + (want_m ? C::M_BYTES : 0));
              if (prm.l2hint) {
                // pass 1's tiles are read again by pass 2 (keep them); pass 2 is their last use
                const uint64_t pol = (pass == 0 && !TP) ? policy_evict_last() : policy_evict_first();
                tma_load_3d_hint(smem + C::OFF_P + ps * C::P_BYTES, &tm_P, &PM_full[ps], c * BN, mb * BM, bhl, pol);
                if (want_m)
                  tma_load_3d_hint(smem + C::OFF_M + ps * C::M_BYTES, &tm_M, &PM_full[ps], c * BN, mb * BM, bhl, pol);
              } else {
                tma_load_3d(smem + C::OFF_P + ps * C::P_BYTES, &tm_P, &PM_full[ps], c * BN, mb * BM, bhl);
                if (want_m) tma_load_3d(smem + C::OFF_M + ps * C::M_BYTES, &tm_M, &PM_full[ps], c * BN, mb * BM, bhl);
              }
              // pass 2 re-reads this unit from L2, which leaves HBM idle for this CTA: pull
              // the same chunk of the CTA's next unit into L2 meanwhile, so that unit's
              // pass 1 finds it there
              if (pass == 1 && prm.l2pf && u + ncl < n_units) {
                const int un = u + ncl, bn_ = un / n_mb, mbn = un - bn_ * n_mb;
                tma_prefetch_l2_3d(&tm_P, c * BN, mbn * BM, bn_);
                tma_prefetch_l2_3d(&tm_M, c * BN, mbn * BM, bn_);
              }
            }
          } else {
            // 16-byte cp.async of the aligned words covering each row segment: 9 for P,
            // 5 for the mask.  Warp 2 takes rows 0..63, warp 3 rows 64..127; lane =
            // (row offset lane/8, word lane%8) so 4 rows go per step and the row start
            // advances by an add.  Words past the tensor's end (rounded up to 16 bytes)
            // are skipped; their columns are masked by the consumers.
            const uint32_t pdst = smem_u32(smem + C::OFF_P + ps * C::P_BYTES);
            const uint32_t mdst = smem_u32(smem + C::OFF_M + ps * C::M_BYTES);
            const int w = int(lane & 7);
            const int r0 = (warp == 2 ? 0 : BM / 2) + int(lane >> 3);
            const int rows = min(BM / 2, sq - mb * BM - (warp == 2 ? 0 : BM / 2));
            unsigned long long el = ((unsigned long long)bhl * sq + mb * BM + r0) * skv + (unsigned long long)c * BN;
            const unsigned long long step = 4ull * skv;
            for (int k = 0; 4 * k + int(lane >> 3) < rows; ++k, el += step) {
              const int r = r0 + 4 * k;
              const unsigned long long sp = ((el * 2) & ~15ull) + 16ull * w;
              const unsigned long long sm_ = (el & ~15ull) + 16ull * w;
              if (sp < prm.p_end16) cp_async16(pdst + r * C::P_PITCH + w * 16, prm.P + sp);
              if (w == 0 && sp + 128 < prm.p_end16) cp_async16(pdst + r * C::P_PITCH + 128, prm.P + sp + 128);
              if (w < 5 && sm_ < prm.m_end16) cp_async16(mdst + r * C::M_PITCH + w * 16, prm.M + sm_);
            }
            cp_async_arrive_noinc(&PM_full[ps]);
          }
          ++pi;
        }
      }
    }
  pm_done:
    if (RAG) cp_async_wait_all();
    if (lane == 0 && warp == 2) {
      for (uint32_t k = 0; k < uint32_t(PST) && k < pi; ++k) {
        const uint32_t i = pi - 1 - k;
        mbar_drain(&PM_full[i % PST], (i / PST) & 1, err, 0x0113);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (lane 0 issues)
    constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, false, false);
    uint32_t job = 0, vi = 0, di = 0;
    for (int u = cid; u < n_units; u += ncl) {
      const int db = di % DOBUF;
      if (!warp_wait(&dO_full[db], (di / DOBUF) & 1, abort_flag, err, 0x0201)) goto mma_done;
      if (CLS) fence_proxy_async_smem();   // class rows: dO arrived by cp.async (generic proxy)
      const uint32_t a_base = smem_u32(smem + C::OFF_DO + db * DO_BYTES);
      for (int pass = 0; pass < npass_mma; ++pass) {
        for (int cl = 0; cl < nloc; ++cl) {
          (void)c0;  // chunk coordinates are not needed by the MMA (V chunk order matches)
          const int slot = job % NSLOT;
          if (!warp_wait(&T_empty[slot], ((job / NSLOT) & 1) ^ 1, abort_flag, err, 0x0202)) goto mma_done;
          const int vs = vi % VST;
          if (!warp_wait(&V_full[vs], (vi / VST) & 1, abort_flag, err, 0x0203)) goto mma_done;
          tc_fence_after();
          if (lane == 0) {
            const uint32_t b_base = smem_u32(smem + C::OFF_V + vs * V_BYTES);
            const uint32_t d_tmem = tmem_base + slot * SLOTC;
#pragma unroll
            for (int kk = 0; kk < kHeadDim / 16; ++kk) {
              // 16 bf16 = 32 B step inside the 128 B swizzle atom; 64-column halves 16 KB / 8 KB apart
              const uint32_t koff = (kk & 3) * 32;
              const uint64_t ad = sdesc_sw128(a_base + (kk >> 2) * (DO_BYTES / 2) + koff, 16, 1024);
              const uint64_t bd = sdesc_sw128(b_base + (kk >> 2) * (V_BYTES / 2) + koff, 16, 1024);
              umma_bf16(d_tmem, ad, bd, idesc, kk > 0 ? 1u : 0u);
            }
            umma_commit(&V_empty[vs]);
            umma_commit(&T_full[slot]);
          }
          __syncwarp();
          ++vi;
          ++job;
        }
      }
      if (lane == 0) umma_commit(&dO_empty[db]);
      __syncwarp();
      ++di;
    }
  mma_done:;
  } else if (warp == 3) {
    // ------------------------------------------------ dS store issuer (aligned rows)
    // Walks the same P/mask stage sequence as the epilogue; for each pass-2 chunk it
    // waits until all epilogue warps wrote dS over the stage, stores it with one TMA
    // tensor store, and frees the stage once the store has read shared memory.
    if constexpr (!RAG && TP) {
      // kTmemP: dS of pass-2 chunk n is written into staging tile n % 2
      uint32_t n = 0;
      bool tp_pend = false;   // class rows: a TMA store of the previous tile may be reading it
      for (int u = cid; u < n_units; u += ncl) {
        const int bhl = CLS ? 0 : u / n_mb, mb = CLS ? 0 : u - bhl * n_mb;
        ClsUnit cu;
        if constexpr (CLS) cu = cls_unit(u, prm);
        for (int cl = 0; cl < nloc; ++cl, ++n) {
          const int c = c0 + cl;
          const int b = n & 1;
          if (!warp_wait(&dS_ready[b], (n >> 1) & 1, abort_flag, err, 0x0306)) goto store_done_tp;
          if constexpr (CLS) {
            // plain stores here (kTmemP with class rows is only reached when forced); the
            // previous tile's TMA store, if any, is waited for first
            if (lane == 0 && n > 0) {
              bulk_wait_read0();
              if (tp_pend) mbar_arrive(&dS_free[b ^ 1]);
            }
            tp_pend = false;
            __syncwarp();
            if (!cls_tma_store_ok(cu, c, prm)) {
              cls_store_chunk(smem_u32(smem + C::OFF_DST + b * (BM * BN * 2)), cu, c, prm, lane);
              __syncwarp();
              if (lane == 0) mbar_arrive(&dS_free[b]);
              continue;
            }
            if (lane == 0) {
              cls_tma_store(&tm_dS, smem + C::OFF_DST + b * (BM * BN * 2), cu, c, skv);
              bulk_commit();
            }
            tp_pend = true;
            __syncwarp();
            continue;
          }
          if (lane == 0) {
            // one store may stay in flight while the epilogue fills the other staging tile
            tma_store_3d(&tm_dS, smem + C::OFF_DST + b * (BM * BN * 2), c * BN, mb * BM, bhl);
            bulk_commit();
            if (n > 0) {
              bulk_wait_read<1>();
              mbar_arrive(&dS_free[b ^ 1]);
            }
          }
          __syncwarp();
        }
      }
    store_done_tp:
      if (lane == 0 && (!CLS || tp_pend)) {
        bulk_wait_read0();
        if (n > 0) mbar_arrive(&dS_free[(n - 1) & 1]);
        bulk_wait_all0();
      }
      __syncwarp();
    } else if constexpr (!RAG) {
      uint32_t pi = 0, dsr_par = 0;
      int npend = 0, pend0 = 0, pend1 = 0;   // stages whose store may still be reading (lane 0)
      for (int u = cid; u < n_units; u += ncl) {
        const int bhl = CLS ? 0 : u / n_mb, mb = CLS ? 0 : u - bhl * n_mb;
        ClsUnit cu;
        if constexpr (CLS) cu = cls_unit(u, prm);
        pi += nloc;  // pass-1 uses of the stages
        for (int cl = 0; cl < nloc; ++cl, ++pi) {
          const int c = c0 + cl;
          const int ps = pi % PST;
          // class rows: a row's first / last chunk is written by the epilogue threads
          // themselves, which also free the stage
          if (CLS && !cls_tma_store_ok(cu, c, prm)) continue;
          if (!warp_wait(&dS_ready[ps], (dsr_par >> ps) & 1u, abort_flag, err, 0x0306)) goto store_done;
          dsr_par ^= 1u << ps;
          if (lane == 0) {
            // keep up to two stores in flight: a stage is freed once its store has read it
            if constexpr (CLS)
              cls_tma_store(&tm_dS, smem + C::OFF_P + ps * C::P_BYTES, cu, c, skv, prm.l2hint != 0);
            else
              if (prm.l2hint)   // dS is not read again: do not let it push P / mask out of L2
                tma_store_3d_hint(&tm_dS, smem + C::OFF_P + ps * C::P_BYTES, c * BN, mb * BM, bhl,
                                  policy_evict_first());
              else
                tma_store_3d(&tm_dS, smem + C::OFF_P + ps * C::P_BYTES, c * BN, mb * BM, bhl);
            bulk_commit();
            if (npend == 2) {
              bulk_wait_read<2>();
              mbar_arrive_cnt(&PM_empty[pend0], kEpiWarps);
              pend0 = pend1;
              pend1 = ps;
            } else if (npend == 1) {
              pend1 = ps;
              npend = 2;
            } else {
              pend0 = ps;
              npend = 1;
            }
          }
          __syncwarp();
        }
        // the next unit's pass 1 may need every stage: release this unit's last stores now
        if (lane == 0 && npend > 0) {
          bulk_wait_read0();
          mbar_arrive_cnt(&PM_empty[pend0], kEpiWarps);
          if (npend == 2) mbar_arrive_cnt(&PM_empty[pend1], kEpiWarps);
          npend = 0;
        }
        __syncwarp();
      }
    store_done:
      if (lane == 0) {
        bulk_wait_read0();
        if (npend >= 1) mbar_arrive_cnt(&PM_empty[pend0], kEpiWarps);
        if (npend == 2) mbar_arrive_cnt(&PM_empty[pend1], kEpiWarps);
        bulk_wait_all0();
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------ epilogue (warps 4..19)
    const int q = warp & 3;               // TMEM lane quadrant (hardware: warp id % 4)
    const int cg = (warp - 4) >> 2;       // column group: chunk columns 16·cg .. +16
    const int row = q * 32 + lane;
    const uint32_t t_lane = uint32_t(q * 32) << 16;
    const int use_mask = prm.use_mask;
    const float scale = prm.scale;
    const uint32_t stg = smem_u32(smem + C::OFF_STG) + (warp - 4) * 32 * C::STG_PITCH;
    uint32_t job = 0, pi = 0, dsn = 0;
    ATTN_BWD_SECT_INIT();
    bool cls_tma_unit = false, cls_row_ok = false;   // class rows: per unit / per thread's row
    int cls_s = 0;                                    // class rows: the unit's window shift

    // Pass 1 of one chunk: row-sum contribution Σ m·dP~·P (the 1/(1-p) is applied once,
    // after the exchange).  kTmemP also parks the masked dP~ and P in TMEM for pass 2.
    auto p1_chunk = [&](unsigned long long row_el, int cl, int cls_s, int mo, float& acc0, float& acc1) -> bool {
      const int c = c0 + cl;
      const int slot = job % NSLOT;
      if (!warp_wait(&T_full[slot], (job / NSLOT) & 1, abort_flag, err, 0x0301)) return false;
      tc_fence_after();
      ATTN_BWD_SECT(0);
      uint32_t v[16];
      tmem_ld16(tmem_base + t_lane + slot * SLOTC + cg * CW, v);
      tmem_wait_ld();
      if (!HOLD) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&T_empty[slot]);
      }
      ++job;
      ATTN_BWD_SECT(1);
      const int ps = pi % PST;
      if (!warp_wait(&PM_full[ps], (pi / PST) & 1, abort_flag, err, 0x0302)) return false;
      ATTN_BWD_SECT(2);
      const unsigned long long el = row_el + (unsigned long long)c * BN;
      uint32_t pw[8], mw[4], mx[4];
      if constexpr (CLS)
        load_row_cls(smem_u32(smem + C::OFF_P + ps * C::P_BYTES), smem_u32(smem + C::OFF_M + ps * C::M_BYTES), row,
                     cg, mo, pw, mw);
      else
        load_row<RAG>(smem_u32(smem + C::OFF_P + ps * C::P_BYTES), smem_u32(smem + C::OFF_M + ps * C::M_BYTES), row,
                      cg, uint32_t(el * 2) & 15u, uint32_t(el) & 15u, pw, mw);
      expand_mask(mw, use_mask, mx);
      ATTN_BWD_SECT(3);
      // valid columns e in [lo, hi) of this thread's 16: ragged rows end inside the last
      // chunk; class windows also start s columns before the row in chunk 0
      int lo = 0, hi = CW;
      if constexpr (RAG) hi = min(max(skv - (c * BN + cg * CW), 0), CW);
      if constexpr (CLS) {
        const int cb = c * BN - cls_s + cg * CW;
        lo = min(max(-cb, 0), CW);
        hi = min(max(skv - cb, 0), CW);
      }
      const bool edge = (RAG || CLS) && (lo > 0 || hi < CW);
      uint32_t m16[8];   // non-TP: 16-bit keep-masks of the 8 bf16 pairs
      if constexpr (TP) {
        if (edge) {
          // columns outside the row hold other rows' bytes
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (e < lo || e >= hi) mw[e >> 2] &= ~(0xFFu << ((e & 3) * 8));
          if (!use_mask) {
#pragma unroll
            for (int i = 0; i < 4; ++i) mx[i] = 0;
#pragma unroll
            for (int e = 0; e < 16; ++e)
              if (e >= lo && e < hi) mx[e >> 2] |= 0xFFu << ((e & 3) * 8);
          } else {
            expand_mask(mw, use_mask, mx);
          }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t m0 = mask_at(mx, 2 * k), m1 = mask_at(mx, 2 * k + 1);
          acc0 = fmaf(__uint_as_float(v[2 * k]), __uint_as_float((pw[k] << 16) & m0), acc0);
          acc1 = fmaf(__uint_as_float(v[2 * k + 1]), __uint_as_float(pw[k] & 0xFFFF0000u & m1), acc1);
          v[2 * k] &= m0;
          v[2 * k + 1] &= m1;
        }
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) m16[k] = use_mask ? mask16_pair(mw, k) : 0xFFFFFFFFu;
        if (edge) {
          // columns outside the row hold other rows' bytes
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (e < lo || e >= hi) m16[e >> 1] &= (e & 1) ? 0x0000FFFFu : 0xFFFF0000u;
        }
        // acc += dP~ * (m * P), both lanes of a pair in one f32x2 FMA (same rounding as two fmaf)
        uint64_t acc = f2(acc0, acc1);
#pragma unroll
        for (int k = 0; k < 8; ++k) acc = f2_fma(f2(v[2 * k], v[2 * k + 1]), bf16x2_to_f2(pw[k] & m16[k]), acc);
        f2_split(acc, acc0, acc1);
      }
      ATTN_BWD_SECT(4);
      // the stage goes back to the producer only after every lane has consumed what it
      // read from it (a release right after the loads let the next fill race them)
      __syncwarp();
      if (lane == 0) mbar_arrive(&PM_empty[ps]);
      if constexpr (TP) {
        // keep what pass 2 needs in TMEM: masked dP~ over the accumulator columns,
        // P (bf16 pairs) in the slot's last 32 columns
        tmem_st16(tmem_base + t_lane + slot * SLOTC + cg * CW, v);
        tmem_st8(tmem_base + t_lane + slot * SLOTC + BN + cg * (CW / 2), pw);
      }
      if constexpr (CP) {
        // masked dP~ as bf16 pairs into this chunk's 32 columns of the compact store
        uint32_t tp[8];
#pragma unroll
        for (int k = 0; k < 8; ++k)
          tp[k] = pack_bf16x2(__uint_as_float(v[2 * k]), __uint_as_float(v[2 * k + 1])) & m16[k];
        tmem_st8(tmem_base + t_lane + C::CP_BASE + cl * (BN / 2) + cg * (CW / 2), tp);
      }
      ATTN_BWD_SECT(5);
      ++pi;
      return true;
    };

    // Row sums of one unit: the four column groups through shared memory (fixed order,
    // deterministic), then -- on a cluster -- the partials of every CTA through
    // distributed shared memory; returns r = Σ dP·P including the 1/(1-p).
    auto exchange = [&](float acc, uint32_t it, float& r) -> bool {
      float* rxb = rx + (it & 1) * 4 * BM;
      rxb[cg * BM + row] = acc;
      mbar_arrive(&pair_bar[q]);
      if (!warp_wait(&pair_bar[q], it & 1, abort_flag, err, 0x0303)) return false;
      r = (rxb[row] + rxb[BM + row]) + (rxb[2 * BM + row] + rxb[3 * BM + row]);
      if (cs > 1) {
        // column group cg serves cluster ranks cg and cg + 4 (itself included)
        const uint32_t slot_addr = smem_u32(xb + ((it & 1) * 8 + rank) * BM + row);
        const uint32_t bar_addr = smem_u32(xbar);
#pragma unroll
        for (int k = cg; k < 8; k += 4) {
          if (k < cs) {
            st_cluster_f32(mapa_shared(slot_addr, k), r);
            mbar_arrive_remote(mapa_shared(bar_addr, k));
          }
        }
        if (!warp_wait_cluster(xbar, it & 1, abort_flag, err, 0x0307)) return false;
        const float* xr = xb + (it & 1) * 8 * BM + row;
        r = 0.f;
        for (int k = 0; k < cs; ++k) r += xr[k * BM];   // same order on every CTA
      }
      r *= scale;
      ATTN_BWD_SECT(6);
      return true;
    };

    // Pass 2 of one chunk: dS = P · (m·dP~/(1-p) − r).
    auto p2_chunk = [&](int bhl, int mb, unsigned long long row_el, int cl, int mo, uint32_t job0, float r) -> bool {
      const int c = c0 + cl;
      uint32_t o[8];
      if constexpr (TP) {
        const int slot = (job0 + cl) % NSLOT;
        uint32_t v[16], pw[8];
        tmem_ld16(tmem_base + t_lane + slot * SLOTC + cg * CW, v);
        tmem_ld8(tmem_base + t_lane + slot * SLOTC + BN + cg * (CW / 2), pw);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&T_empty[slot]);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float p0 = __uint_as_float(pw[k] << 16), p1 = __uint_as_float(pw[k] & 0xFFFF0000u);
          o[k] = pack_bf16x2(p0 * fmaf(__uint_as_float(v[2 * k]), scale, -r),
                             p1 * fmaf(__uint_as_float(v[2 * k + 1]), scale, -r));
        }
        if constexpr (!RAG) {
          const int b = dsn & 1;
          if (!warp_wait(&dS_free[b], ((dsn >> 1) & 1) ^ 1, abort_flag, err, 0x0305)) return false;
          const uint32_t d_row = smem_u32(smem + C::OFF_DST + b * (BM * BN * 2)) + row * 128;
#pragma unroll
          for (int i = 0; i < 2; ++i)
            sts128(d_row + (((cg * 2 + i) ^ (row & 7)) << 4),
                   make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&dS_ready[b]);
        } else {
          store_rag_dS(o, stg, lane, prm, bhl, sq, skv, mb, q, c, cg);
        }
        ++dsn;
        return true;
      } else {
        uint32_t v[16];
        if constexpr (CP) {
          // masked dP~ from the compact store, widened back to fp32 (mask already applied)
          uint32_t tp[8];
          tmem_ld8(tmem_base + t_lane + C::CP_BASE + cl * (BN / 2) + cg * (CW / 2), tp);
          tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            v[2 * k] = tp[k] << 16;
            v[2 * k + 1] = tp[k] & 0xFFFF0000u;
          }
        } else {
          int slot;
          if (RES) {
            slot = (job0 + cl) % NSLOT;
          } else {
            slot = job % NSLOT;
            if (!warp_wait(&T_full[slot], (job / NSLOT) & 1, abort_flag, err, 0x0304)) return false;
            tc_fence_after();
            ++job;
          }
          tmem_ld16(tmem_base + t_lane + slot * SLOTC + cg * CW, v);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&T_empty[slot]);
        }
        ATTN_BWD_SECT(8);
        const int ps = pi % PST;
        if (!warp_wait(&PM_full[ps], (pi / PST) & 1, abort_flag, err, 0x0305)) return false;
        ATTN_BWD_SECT(9);
        const unsigned long long el = row_el + (unsigned long long)c * BN;
        const uint32_t p_stage = smem_u32(smem + C::OFF_P + ps * C::P_BYTES);
        uint32_t pw[8], mw[4], mx[4];
        if constexpr (CP && !RAG) {
          // the compact store holds the masked dP~ and pass 2 loaded no mask: P only
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const uint4 t = lds128(p_stage + row * 128 + (((cg * 2 + i) ^ (row & 7)) << 4));
            pw[4 * i] = t.x; pw[4 * i + 1] = t.y; pw[4 * i + 2] = t.z; pw[4 * i + 3] = t.w;
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) mx[i] = 0xFFFFFFFFu;
          (void)mw;
        } else {
          if constexpr (CLS)
            load_row_cls(p_stage, smem_u32(smem + C::OFF_M + ps * C::M_BYTES), row, cg, mo, pw, mw);
          else
            load_row<RAG>(p_stage, smem_u32(smem + C::OFF_M + ps * C::M_BYTES), row, cg, uint32_t(el * 2) & 15u,
                          uint32_t(el) & 15u, pw, mw);
          expand_mask(mw, use_mask, mx);
        }
        ATTN_BWD_SECT(10);
        // dS = P * (m * dP~ * s - r), pairs in f32x2 (same rounding as the scalar fmaf / mul)
        const uint64_t s2 = f2(scale, scale), nr2 = f2(-r, -r);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          uint32_t t0 = v[2 * k], t1 = v[2 * k + 1];
          if (!CP) {   // kCompact's store already holds the masked dP~
            t0 &= mask_at(mx, 2 * k);
            t1 &= mask_at(mx, 2 * k + 1);
          }
          o[k] = pack_bf16x2_f2(f2_mul(bf16x2_to_f2(pw[k]), f2_fma(f2(t0, t1), s2, nr2)));
        }
        ATTN_BWD_SECT(11);
        if (CLS && !cls_tma_unit_ok(cls_tma_unit, c, cls_s, skv)) {
          // class rows, a row's first / last chunk: this thread's 16 values are two
          // 16-byte aligned words of its row; words crossing the row end go element-wise
          if (cls_row_ok) {
            const int col0 = c * BN - cls_s + cg * CW;
            uint8_t* dst = prm.dS + 2 * (row_el + col0);
#pragma unroll
            for (int w = 0; w < 2; ++w) {
              const int cw = col0 + 8 * w;
              if (cw >= 0 && cw + 8 <= skv) {
                *reinterpret_cast<uint4*>(dst + 16 * w) = make_uint4(o[4 * w], o[4 * w + 1], o[4 * w + 2], o[4 * w + 3]);
              } else {
#pragma unroll
                for (int e = 0; e < 8; ++e)
                  if (cw + e >= 0 && cw + e < skv)
                    reinterpret_cast<unsigned short*>(dst + 16 * w)[e] = (unsigned short)(o[4 * w + (e >> 1)] >> ((e & 1) * 16));
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&PM_empty[ps]);
        } else if constexpr (!RAG) {
          // dS overwrites P in place (same swizzled positions); warp 3 stores the chunk
          const uint32_t p_row = p_stage + row * 128;
#pragma unroll
          for (int i = 0; i < 2; ++i)
            sts128(p_row + (((cg * 2 + i) ^ (row & 7)) << 4),
                   make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&dS_ready[ps]);
          ATTN_BWD_SECT(12);
        } else {
          __syncwarp();
          if (lane == 0) mbar_arrive(&PM_empty[ps]);
          store_rag_dS(o, stg, lane, prm, bhl, sq, skv, mb, q, c, cg);
        }
        ++pi;
        return true;
      }
    };

    {
      uint32_t it = 0;
      for (int u = cid; u < n_units; u += ncl, ++it) {
        const int bhl = CLS ? 0 : u / n_mb, mb = CLS ? 0 : u - bhl * n_mb;
        unsigned long long row_el = CLS ? 0ull : ((unsigned long long)bhl * sq + mb * BM + row) * skv;
        int mo = 0;
        if constexpr (CLS) {
          const ClsUnit cu = cls_unit(u, prm);
          cls_s = cu.s;
          mo = q >= 2 ? cu.mo[1] : cu.mo[0];   // TMEM lanes 0..63: sub-class A, 64..127: B
          cls_tma_unit = !cu.pad && !cu.fallback;
          const int rho = (q >= 2 ? cu.rho[1] : cu.rho[0]) + 16 * (row & 63);
          cls_row_ok = rho < kGroups * sq;
          row_el = (unsigned long long)(cu.g0 + rho) * skv;   // flat element index of the row start
        }
        const uint32_t job0 = job;
        float acc0 = 0.f, acc1 = 0.f, r;
        for (int cl = 0; cl < nloc; ++cl)
          if (!p1_chunk(row_el, cl, cls_s, mo, acc0, acc1)) goto epi_done;
        if (TP || CP) tmem_wait_st();
        if (!exchange(acc0 + acc1, it, r)) goto epi_done;
        for (int cl = 0; cl < nloc; ++cl)
          if (!p2_chunk(bhl, mb, row_el, cl, mo, job0, r)) goto epi_done;
      }
    }
  epi_done:
    ATTN_BWD_SECT_FLUSH();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (prm.cs > 1) cluster_sync();   // no CTA leaves while a peer may still write into its shared memory
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TSLOTS * BN);
  }
  ATTN_BWD_WAIT_STATS_END();
}

}  // namespace ds
}  // namespace attn_bwd
