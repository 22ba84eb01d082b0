// dv_kernel.cuh — fused dV kernel: dV[b,kvh] = Σ_{g<10} P_dropᵀ[b,10·kvh+g] · dO[b,:,10·kvh+g,:]
// on tcgen05, with the sum over the 10 grouped query heads folded into the
// K loop (K = 10 · seq_q), so no [bs,80,skv,128] expansion ever exists.
//
// Reference math: attn_bwd/starting_point.py:61-68 (dV_exp = P̃ᵀ·dO, then the
// group sum and the bf16 cast).
//
// Work unit: one (batch, kv-head, 128-row tile of seq_kv).  Both operands are
// MN-major in shared memory: A = P_drop tile [64 seq_q rows][128 seq_kv cols]
// (seq_kv contiguous), B = dO tile [64 seq_q rows][128 d] read in place from
// [bs, sq, 80, 128] (row stride 80·128·2 B).  The accumulator [128 x 128] f32
// lives in TMEM, double-buffered across units so the epilogue of one unit
// overlaps the MMAs of the next.
//
// Roles: warp 0 producer, warp 1 MMA issuer + TMEM owner, warps 2..5 epilogue
// (warp w drains TMEM lanes 32·(w%4)..); ragged rows add warps 6..13 (re-align) and
// warp 14 (raw P_drop producer).
//
// Row formats (template flag RAG):
//   RAG = false  seq_kv % 8 == 0: P_drop tiles are TMA tensor tiles (128B swizzle).
//   RAG = true   any seq_kv: P_drop rows are not 16-byte aligned.  Rows 8 apart are
//                16·seq_kv bytes apart, a 16-byte multiple, so each residue class of
//                rows mod 8 is a legal 2-D tensor: the producer fetches the 64 rows of
//                a K chunk as 8 TMA boxes (one per class, 8 rows x 272 B from the
//                16-byte boundary below each row's 128-column segment), and warps
//                6..13 re-align the bytes in registers and write the 128B-swizzled
//                MN-major tile the MMA reads (zeroing columns >= seq_kv and rows >=
//                seq_q).  The last partial group of 8 rows of the buffer (outside
//                the class tensor) is fetched by 16-byte cp.async instead.
#pragma once
#include "sm100.cuh"

namespace attn_bwd {
namespace dv {
constexpr int BM = 128;   // seq_kv rows per unit
constexpr int BK = 64;    // seq_q rows per K chunk
constexpr int A_BYTES = BK * BM * 2;          // 16 KB (two 64-col MN blocks of 8 KB)
constexpr int B_BYTES = BK * kHeadDim * 2;    // 16 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;

// FPM (aligned rows only): P_drop is not read; each K chunk's A tile is formed in shared
// memory from attn_weights and the dropout mask as bf16(P · m · 1/(1-p)), the identity by
// which the reference's inputs are made (eval_modal_attn_bwd.py:159-161).  Warps 6..13 convert
// a stage in place once its P and mask tiles have landed.
template <bool RAG, bool FPM = false>
struct Cfg {
  static constexpr int kThreads = RAG ? 480 : FPM ? 448 : 192;   // RAG: + 8 re-align warps (6..13), raw producer (14)
  static constexpr int ST = RAG ? 4 : FPM ? 5 : 6;     // operand stages (RAG: 3 + 6 raw measured slower)
  static constexpr int MSK_BYTES = FPM ? BK * BM : 0;  // FPM: mask tile per stage (64 rows x 128 B, SW128)
  static constexpr int A_READY = 8;                    // warps that arrive on a_ready (re-align / convert)
  static constexpr int RST = RAG ? 4 : 0;              // raw P_drop row stages
  static constexpr int RAW_PITCH = 272;                // 256 B of row + 16 B of misalignment slack
  static constexpr int CLS_BYTES = 8 * RAW_PITCH;      // one class box: 8 rows (2176 B, 128-byte multiple)
  static constexpr int RAW_BYTES = BK * RAW_PITCH;
  static constexpr int OFF_MSK = ST * STAGE_BYTES;
  static constexpr int OFF_RAW = OFF_MSK + ST * MSK_BYTES;
  static constexpr int OFF_BAR = OFF_RAW + RST * RAW_BYTES;
  static constexpr int NBAR = 3 * ST + 2 * RST + 4;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 64 + 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "dV kernel shared memory");
};

struct Params {
  int sq, skv;
  int n_units;     // local (batch, kv-head) count × seq_kv tiles
  int n_jt;        // seq_kv tiles per (batch, kv-head)
  int n_kc;        // seq_q chunks per head
  int unit_base;   // global (batch·8 + kv-head) index of local unit 0
  int* err;
  const uint8_t* Pd;              // local P_drop base (RAG path)
  unsigned long long pd_end16;    // bytes of P_drop rounded up to 16
  long long tma_rows;             // RAG: rows covered by the class tensor map (8 · floor(rows / 8))
  float scale;                    // FPM: 1 / (1 - p)
};

// out[j] = bytes [4j+sh, 4j+sh+4) of the little-endian stream `in` (NOUT+4 words).
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

// Shared-memory row of logical row r (0..63) of a raw stage: class box r % 8, row r / 8.
__device__ __forceinline__ int raw_row(int r) { return (r & 7) * 8 + (r >> 3); }

// Fallback for K chunks that reach the buffer's last partial group of 8 rows: 16-byte
// cp.async of the 17 aligned words covering each row's 128-column segment, into the
// same layout the class boxes produce, then a wait for completion.  Words past the
// tensor's end (rounded up to 16 bytes) are skipped; the re-align warps zero those
// columns.
__device__ __forceinline__ void raw_rows_sync(uint32_t rdst, const Params& prm, int bhl, int kc, int jt,
                                              uint32_t lane) {
  const int rows = min(BK, prm.sq - kc * BK);
  for (int f = int(lane); f < rows * 17; f += 32) {
    const int r = f / 17, w = f - r * 17;
    const unsigned long long el = ((unsigned long long)bhl * prm.sq + kc * BK + r) * prm.skv + (unsigned long long)jt * BM;
    const unsigned long long src = ((el * 2) & ~15ull) + 16ull * w;
    if (src < prm.pd_end16) sm100::cp_async16(rdst + raw_row(r) * 272 + w * 16, prm.Pd + src);
  }
  sm100::cp_async_wait_all();
}

template <bool RAG, bool FPM = false>
__global__ void __launch_bounds__(Cfg<RAG, FPM>::kThreads, 1)
dv_kernel(const __grid_constant__ CUtensorMap tm_Pd,   // aligned: (skv, sq, bh_local) box (64,64,1) SW128;
                                                       // RAG: u32 (4·skv, rows/8) box (68, 8), no swizzle;
                                                       // FPM: attn_weights, as aligned
          const __grid_constant__ CUtensorMap tm_dO,   // (d, h, s, b)         box (64,1,64,1) SW128
          __nv_bfloat16* __restrict__ dV,              // local [units, skv, 128]
          const Params prm,
          const __grid_constant__ CUtensorMap tm_M) {  // FPM: mask u8 (skv, sq, bh_local) box (128,64,1) SW128
  using namespace sm100;
  using C = Cfg<RAG, FPM>;
  static_assert(!(RAG && FPM), "P_drop from P and mask: aligned rows only");
  constexpr int ST = C::ST, RST = C::RST;
  constexpr int RSTD = RST > 0 ? RST : 1;  // keeps the (unused) ragged arithmetic defined when RST == 0
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = bars + ST;
  uint64_t* a_ready = bars + 2 * ST;      // RAG: the 4 re-align warps wrote the A tile
  uint64_t* raw_full = a_ready + ST;
  uint64_t* raw_empty = raw_full + RST;
  uint64_t* acc_full = raw_empty + RST;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  ATTN_BWD_WAIT_STATS_BEGIN();
  const uint32_t warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); mbar_init(&a_ready[i], C::A_READY); }
    // raw_full: the producer's lane 0 (with the class boxes' bytes as transaction count)
    for (int i = 0; i < RST; ++i) { mbar_init(&raw_full[i], 1); mbar_init(&raw_empty[i], 8); }
    for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], 4); }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    if (!RAG || prm.tma_rows > 0) prefetch_tmap(&tm_Pd);
    prefetch_tmap(&tm_dO);
    if (FPM) prefetch_tmap(&tm_M);
  }
  if (warp == 1) { tmem_alloc(tmem_base_slot, 256); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;
  const int n_units = prm.n_units, n_jt = prm.n_jt, n_kc = prm.n_kc;
  int* err = prm.err;

  if (warp == 0) {
    uint32_t si = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
      const int ul = u / n_jt, jt = u - ul * n_jt;
      const int ug = prm.unit_base + ul;
      const int b = ug / kKvHeads, kvh = ug - b * kKvHeads;
      for (int g = 0; g < kGroups; ++g) {
        const int h = kvh * kGroups + g;
        const int bhl = ul * kGroups + g;
        for (int kc = 0; kc < n_kc; ++kc) {
          const int s = si % ST;
          if (!warp_wait(&empty[s], ((si / ST) & 1) ^ 1, abort_flag, err, 0x1101)) goto prod_done;
          if (lane == 0) {
            {
              uint8_t* a = smem + s * STAGE_BYTES;
              uint8_t* bsm = a + A_BYTES;
              mbar_arrive_expect_tx(&full[s], RAG ? B_BYTES : STAGE_BYTES + C::MSK_BYTES);
              if (!RAG) {
                tma_load_3d(a, &tm_Pd, &full[s], jt * BM, kc * BK, bhl);
                tma_load_3d(a + A_BYTES / 2, &tm_Pd, &full[s], jt * BM + 64, kc * BK, bhl);
              }
              if (FPM) tma_load_3d(smem + C::OFF_MSK + s * C::MSK_BYTES, &tm_M, &full[s], jt * BM, kc * BK, bhl);
              tma_load_4d(bsm, &tm_dO, &full[s], 0, h, kc * BK, b);
              tma_load_4d(bsm + B_BYTES / 2, &tm_dO, &full[s], 64, h, kc * BK, b);
            }
          }
          ++si;
        }
      }
    }
  prod_done:
    if (lane == 0) {
      for (uint32_t k = 0; k < uint32_t(ST) && k < si; ++k) {
        const uint32_t i = si - 1 - k;
        mbar_drain(&full[i % ST], (i / ST) & 1, err, 0x1111);
      }

    }
    __syncwarp();
  } else if (warp == 1) {
    constexpr uint32_t idesc = idesc_bf16_f32(BM, kHeadDim, true, true);
    uint32_t si = 0, ui = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++ui) {
      const int acc = ui & 1;
      if (!warp_wait(&acc_empty[acc], ((ui >> 1) & 1) ^ 1, abort_flag, err, 0x1201)) goto mma_done;
      tc_fence_after();
      {
        const uint32_t d_tmem = tmem_base + acc * kHeadDim;
        const int nk = kGroups * n_kc;
        for (int k = 0; k < nk; ++k) {
          const int s = si % ST;
          if (!warp_wait(&full[s], (si / ST) & 1, abort_flag, err, 0x1202)) goto mma_done;
          if ((RAG || FPM) && !warp_wait(&a_ready[s], (si / ST) & 1, abort_flag, err, 0x1203)) goto mma_done;
          tc_fence_after();
          if (lane == 0) {
            const uint32_t a = smem_u32(smem + s * STAGE_BYTES);
            const uint32_t bsm = a + A_BYTES;
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              // 16 k-rows = two 8-row swizzle atoms = 2048 B
              const uint64_t ad = sdesc_sw128(a + kk * 2048, A_BYTES / 2, 1024);
              const uint64_t bd = sdesc_sw128(bsm + kk * 2048, B_BYTES / 2, 1024);
              umma_bf16(d_tmem, ad, bd, idesc, (k > 0 || kk > 0) ? 1u : 0u);
            }
            umma_commit(&empty[s]);
          }
          __syncwarp();
          ++si;
        }
        if (lane == 0) umma_commit(&acc_full[acc]);
        __syncwarp();
      }
    }
  mma_done:;
  } else if (warp < 6) {
    // epilogue warps 2..5
    const int q = warp & 3;
    const uint32_t t_lane = uint32_t(q * 32) << 16;
    const int skv = prm.skv;
    uint32_t ui = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++ui) {
      const int ul = u / n_jt, jt = u - ul * n_jt;
      const int acc = ui & 1;
      if (!warp_wait(&acc_full[acc], (ui >> 1) & 1, abort_flag, err, 0x1301)) break;
      tc_fence_after();
      const int j = jt * BM + q * 32 + lane;
      __nv_bfloat16* out = dV + (size_t(ul) * skv + j) * kHeadDim;
#pragma unroll
      for (int cc = 0; cc < kHeadDim / 32; ++cc) {
        uint32_t v[32];
        __syncwarp();
        tmem_ld32(tmem_base + t_lane + acc * kHeadDim + cc * 32, v);
        tmem_wait_ld();
        if (j < skv) {
          uint4* o = reinterpret_cast<uint4*>(out + cc * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[i * 8 + 0]), __uint_as_float(v[i * 8 + 1]));
            w.y = pack_bf16x2(__uint_as_float(v[i * 8 + 2]), __uint_as_float(v[i * 8 + 3]));
            w.z = pack_bf16x2(__uint_as_float(v[i * 8 + 4]), __uint_as_float(v[i * 8 + 5]));
            w.w = pack_bf16x2(__uint_as_float(v[i * 8 + 6]), __uint_as_float(v[i * 8 + 7]));
            o[i] = w;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
  }

  else if (FPM) {
    // convert warps 6..13: A tile (P, two 64-column SW128 halves of 64 rows) -> P_drop in place.
    // 16-byte chunk c (8 columns) of row r sits at chunk c ^ (r % 8); its 8 mask bytes are the
    // low or high half of mask chunk (4·half + c/2) of the same row (128 B rows, SW128).
    const int t = int(threadIdx.x) - 6 * 32;   // 0..255
    const uint64_t s2 = f2(prm.scale, prm.scale);
    uint32_t si = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
      for (int g = 0; g < kGroups; ++g) {
        for (int kc = 0; kc < n_kc; ++kc, ++si) {
          const int s = si % ST;
          if (!warp_wait(&full[s], (si / ST) & 1, abort_flag, err, 0x1501)) goto convert_done;
          const uint32_t a = smem_u32(smem + s * STAGE_BYTES);
          const uint32_t mk = smem_u32(smem + C::OFF_MSK + s * C::MSK_BYTES);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int f = t + 256 * i;          // 1024 chunks: (half, row, chunk)
            const int hf = f >> 9, r = (f >> 3) & 63, c = f & 7;
            const uint32_t pa = a + hf * (A_BYTES / 2) + r * 128 + ((c ^ (r & 7)) << 4);
            const int q = 4 * hf + (c >> 1);
            uint32_t mw[2];
            asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];" : "=r"(mw[0]), "=r"(mw[1])
                         : "r"(mk + r * 128 + ((q ^ (r & 7)) << 4) + (c & 1) * 8));
            const uint4 pv = lds128(pa);
            uint32_t w[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              // bf16 pair k (elements 2k, 2k+1): mask bytes 2k, 2k+1 of the 8
              const uint32_t m16 = __byte_perm(mw[k >> 1], 0u, (k & 1) ? 0x4342u : 0x4140u) * 0xFFFFu;
              w[k] = pack_bf16x2_f2(f2_mul(bf16x2_to_f2(w[k]), s2)) & m16;
            }
            sts128(pa, make_uint4(w[0], w[1], w[2], w[3]));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_ready[s]);
        }
      }
    }
  convert_done:;
  }
  else if (RAG && warp == 14) {
    // raw P_drop producer: runs up to RST K chunks ahead of the re-align warps, independent
    // of the operand ring (which waits for the MMA)
    uint32_t ri = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
      const int ul = u / n_jt, jt = u - ul * n_jt;
      for (int g = 0; g < kGroups; ++g) {
        const int bhl = ul * kGroups + g;
        for (int kc = 0; kc < n_kc; ++kc, ++ri) {
          const int rs = ri % RSTD;
          if (!warp_wait(&raw_empty[rs], ((ri / RSTD) & 1) ^ 1, abort_flag, err, 0x1102)) goto raw_done;
          uint8_t* rdst = smem + C::OFF_RAW + rs * C::RAW_BYTES;
          const long long r0 = (long long)bhl * prm.sq + kc * BK;
          if (r0 + min(BK, prm.sq - kc * BK) <= prm.tma_rows) {
            if (lane == 0) mbar_arrive_expect_tx(&raw_full[rs], C::RAW_BYTES);
            __syncwarp();
            if (lane < 8) {
              // class box `lane`: rows r0 + lane + 8i, i < 8 (row k of its 8-row group)
              const long long rm = r0 + lane;
              const unsigned long long off =
                  ((unsigned long long)(rm & 7) * 2 * prm.skv + (unsigned long long)jt * 256) & ~15ull;
              tma_load_2d(rdst + lane * C::CLS_BYTES, &tm_Pd, &raw_full[rs], int(off >> 2), int(rm >> 3));
            }
          } else {
            raw_rows_sync(smem_u32(rdst), prm, bhl, kc, jt, lane);
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_full[rs]);
          }
        }
      }
    }
  raw_done:
    if (lane == 0) {
      for (uint32_t k = 0; k < uint32_t(RSTD) && k < ri; ++k) {
        const uint32_t i = ri - 1 - k;
        mbar_drain(&raw_full[i % RSTD], (i / RSTD) & 1, err, 0x1112);
      }
    }
    __syncwarp();
  }
  else if (RAG) {
    // re-align warps 6..13: thread t handles one row r of the chunk and the 32-column
    // quarter qt = t / 64 (uniform per warp) of the 128-column tile.  Rows go diagonally
    // over each group of 8 threads (i = t % 8, class m = (i + t/8) % 8, r = m + 8i), so
    // both the raw-row reads (row 8m + i) and the swizzled writes (chunk ^ m) of a
    // quarter-warp fall in 8 different 16-byte bank groups.
    const int t = int(threadIdx.x) - 6 * 32;
    const int qt = t >> 6;
    const int ci = t & 7, cm = (ci + ((t >> 3) & 7)) & 7;
    const int r = cm + 8 * ci;
    const int sq = prm.sq, skv = prm.skv;
    uint32_t si = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
      const int ul = u / n_jt, jt = u - ul * n_jt;
      const int nvalid = min(max(skv - (jt * BM + qt * 32), 0), 32);
      for (int g = 0; g < kGroups; ++g) {
        const int bhl = ul * kGroups + g;
        for (int kc = 0; kc < n_kc; ++kc, ++si) {
          const int s = si % ST, rs = si % RSTD;
          if (!warp_wait(&raw_full[rs], (si / RSTD) & 1, abort_flag, err, 0x1401)) goto realign_done;
          if (!warp_wait(&empty[s], ((si / ST) & 1) ^ 1, abort_flag, err, 0x1402)) goto realign_done;
          const int srow = kc * BK + r;
          uint32_t w[16];
          if (srow < sq) {
            const unsigned long long el = ((unsigned long long)bhl * sq + srow) * skv + (unsigned long long)jt * BM;
            const uint32_t src = smem_u32(smem + C::OFF_RAW + rs * C::RAW_BYTES + raw_row(r) * C::RAW_PITCH + qt * 64);
            uint32_t in[20];
#pragma unroll
            for (int i = 0; i < 5; ++i) {
              const uint4 x = lds128(src + i * 16);
              in[4 * i] = x.x; in[4 * i + 1] = x.y; in[4 * i + 2] = x.z; in[4 * i + 3] = x.w;
            }
            byte_shift<16>(in, uint32_t(el * 2) & 15u, w);
            if (nvalid < 32) {   // last, partial tile only: columns >= seq_kv belong to the next row
#pragma unroll
              for (int k = 0; k < 16; ++k) {
                if (2 * k >= nvalid) w[k] = 0;
                else if (2 * k + 1 >= nvalid) w[k] &= 0xFFFFu;
              }
            }
          } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) w[k] = 0;
          }
          // 128B-swizzled MN-major row: 16-byte chunk k of row r sits at chunk k ^ (r % 8)
          const uint32_t dst = smem_u32(smem + s * STAGE_BYTES + (qt >> 1) * (A_BYTES / 2) + r * 128);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int k = (qt & 1) * 4 + i;
            sts128(dst + ((k ^ (r & 7)) << 4), make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&raw_empty[rs]);
            mbar_arrive(&a_ready[s]);
          }
        }
      }
    }
  realign_done:;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 256);
  }
  ATTN_BWD_WAIT_STATS_END();
}

}  // namespace dv
}  // namespace attn_bwd
