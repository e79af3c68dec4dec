// Causal sliding-window prefill on the sm_100a tensor cores (tcgen05 + TMEM).
//
// Reference: local_causal_prefill_kernel (triton_local_prefill.py:17-58), one program
// per query row scanning keys [i-W+1, i] with an online softmax.  Here a persistent CTA
// per SM walks work items round-robin; an item is two 128-row query tiles of one (b, h),
// and the CTA streams the 128-key tiles that intersect their windows (W/128 + 2 tiles for
// W a multiple of 128).  Barrier phases, the K/V ring and TMEM carry over from item to
// item, so one item's Q load, first products and write-out overlap its neighbours:
//
//   warp 0      TMA producer: each item's Q tiles (Q_t reloads as soon as the last S_t
//               product of the previous item has completed), then K and V tiles into two
//               STAGES-deep rings with separate full/empty barriers: K(j) is released as soon as
//               both S(j) products complete, so K(j+2) streams in while V(j) is still
//               being multiplied (about one KV-tile period of lead instead of none)
//   warp 1      MMA issuer (whole warp, one elected lane issues): S_t = Q_t K^T (SS
//               form, both operands in shared memory, K-major), O_t += P_t V (TS form:
//               P read from TMEM, V from shared memory, MN-major)
//   warps 4-7   softmax of query tile 0, warps 8-11 of query tile 1: thread = row =
//               TMEM lane (warp w reaches lanes [32*(w%4), 32*(w%4)+32)); a thread holds
//               its 128 scores in registers (setmaxnreg gives the softmax warpgroups 184
//               registers and the control warpgroup 128)
//   warps 2-3   idle
//
// TMEM (512 columns): S_0 [0,128), S_1 [128,256), O_0 [256,256+D), O_1 [384,384+D).
// P_t (bf16 pairs) overwrites the first 64 columns of S_t once S_t is in registers, in two
// halves (keys 0-63, then 64-127) with a barrier each, so the PV product of the first half
// runs while the softmax warps compute the second.
// The MMA warp interleaves O_0(j), S_0(j+1), O_1(j), S_1(j+1), so the softmax of one
// tile overlaps the other tile's tensor-core work.  The running max is only moved
// (and O rescaled in TMEM) when a tile's max exceeds it by more than 2^8.  Key tiles cut
// by the causal diagonal, the window start or the sequence end are masked in registers
// (scores out of range become -inf before the row max); exponentials run on MUFU.
//
// Keys are indexed in the concatenation [halo ; keys] (halo_len a multiple of 128):
// query i sits at position i + halo_len and sees positions (i+halo-W, i+halo].
#pragma once

#include <algorithm>

#include "prefill_generic.cuh"

namespace spa {

constexpr int kPfTile = 128;
constexpr int kPfStages = 2;
constexpr int kPfThreads = 384;
constexpr int kPfRegsCtl = 128;      // warps 0-3 (TMA, MMA, idle) after setmaxnreg.dec
constexpr int kPfRegsSoftmax = 184;  // warps 4-11 after setmaxnreg.inc
static_assert(128 * kPfRegsCtl + 256 * kPfRegsSoftmax <= kPfThreads * 168, "register split exceeds the launch");
static_assert(kPfRegsCtl + 2 * kPfRegsSoftmax <= 512, "register split exceeds a sub-partition");
constexpr float kPfRescaleThreshold = 8.0f;  // log2 units

struct PfTcArgs {
  void* out;
  int S, W, halo, row0, row1, H, n_pairs, n_items;  // item = (query-tile pair, b*H + h)
  float scale_log2;
};

template <int D>
struct PfSmem {
  static constexpr int kBoxBytes = kPfTile * 128;  // [128 rows x 64 elements] bf16
  static constexpr int kBoxes = D / 64;
  static constexpr int kTileBytes = kBoxes * kBoxBytes;
  static constexpr int kQ0 = 0;
  static constexpr int kQ1 = kTileBytes;
  static constexpr int kK = 2 * kTileBytes;
  static constexpr int kV = kK + kPfStages * kTileBytes;
  // epilogue staging: per softmax warp 32 rows x 32 output columns (16-bit), rows padded
  // to 80 bytes so the row-wise writes and the column-wise reads avoid bank conflicts
  static constexpr int kStageRow = 80;
  static constexpr int kStage = kV + kPfStages * kTileBytes;
  static constexpr int kStageBytes = 8 * 32 * kStageRow;
  static constexpr int kBar = kStage + kStageBytes;
  // barriers: q_full[2], k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], p_half[2],
  // p_full[2], o_final[2], mma_done, q_empty[2], o_empty[2]; + tmem slot
  static constexpr int kNumBars = 2 + 4 * kPfStages + 2 + 2 + 2 + 2 + 1 + 2 + 2;
  static constexpr int kBytes = kBar + kNumBars * 8 + 16 + 1024;
};

// ---- tcgen05 wrappers
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                       uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

#define SPA_TMEM_LD32(taddr, r)                                                                                  \
  asm volatile(                                                                                                  \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"   \
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                                        \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),         \
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),  \
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), \
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])  \
      : "r"(taddr))

#define SPA_TMEM_ST32(taddr, r)                                                                                  \
  asm volatile(                                                                                                  \
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"   \
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),                         \
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),        \
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),           \
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),          \
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])                      \
      : "memory")

#define SPA_TMEM_ST16(taddr, r)                                                                                  \
  asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14," \
               "%15,%16};" ::"r"(taddr),                                                                        \
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),          \
               "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])     \
               : "memory")

#define SPA_TMEM_LD16(taddr, r)                                                                                  \
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];" \
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),  \
                 "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),        \
                 "=r"(r[15])                                                                                     \
               : "r"(taddr))

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor (SWIZZLE_128B, sm_100 version field = 1).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= 1ull << 46;  // version
  d |= 2ull << 61;  // SWIZZLE_128B
  return d;
}

// kind::f16 instruction descriptor: fp32 accumulate, A/B 16-bit (fmt 0 = f16, 1 = bf16).
__host__ __device__ constexpr uint32_t instr_desc_f16(int fmt, int m, int n, int a_mn_major, int b_mn_major) {
  return (1u << 4) | (static_cast<uint32_t>(fmt) << 7) | (static_cast<uint32_t>(fmt) << 10) |
         (static_cast<uint32_t>(a_mn_major) << 15) | (static_cast<uint32_t>(b_mn_major) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

template <typename T>
struct PfFmt;
template <>
struct PfFmt<__nv_bfloat16> {
  static constexpr int kFmt = 1;
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};
template <>
struct PfFmt<__half> {
  static constexpr int kFmt = 0;
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

// Key-tile range [lo, hi] (concatenated coordinates) of query tile qt; empty if lo > hi.
__device__ __forceinline__ void pf_tile_range(const PfTcArgs& a, int qt, int& lo, int& hi) {
  const int qc0 = qt * kPfTile + a.halo;                          // first query position
  const int qlast = min(qt * kPfTile + kPfTile, a.S) - 1 + a.halo;  // last real query position
  const int first_key = qc0 - a.W + 1;
  lo = first_key <= 0 ? 0 : first_key / kPfTile;
  hi = qlast / kPfTile;
}

// One work item of the persistent kernel: a pair of query tiles of one (b, h).
struct PfItem {
  int qt0, bh, J0, J1;
  int lo[2], hi[2];
  bool act[2];
};
__device__ __forceinline__ PfItem pf_item(const PfTcArgs& a, int w) {
  PfItem I;
  const int p = w % a.n_pairs;
  I.bh = w / a.n_pairs;
  I.qt0 = a.row0 / kPfTile + 2 * p;
  const int last_tile = (a.row1 - 1) / kPfTile;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    I.act[t] = I.qt0 + t <= last_tile;
    pf_tile_range(a, I.qt0 + t, I.lo[t], I.hi[t]);
    if (I.lo[t] > I.hi[t]) I.act[t] = false;
  }
  I.J0 = I.act[0] ? I.lo[0] : I.lo[1];
  I.J1 = I.act[1] ? I.hi[1] : I.hi[0];
  return I;
}

template <typename T, int D>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap khmap,
                      const __grid_constant__ CUtensorMap vhmap, const PfTcArgs a) {
  using L = PfSmem<D>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars;  // [2] Q_t of the current item loaded
  uint64_t* k_full = bars + 2;
  uint64_t* k_empty = k_full + kPfStages;
  uint64_t* v_full = k_empty + kPfStages;
  uint64_t* v_empty = v_full + kPfStages;
  uint64_t* s_full = v_empty + kPfStages;
  uint64_t* p_half = s_full + 2;
  uint64_t* p_full = p_half + 2;
  uint64_t* o_final = p_full + 2;
  uint64_t* mma_done = o_final + 2;
  uint64_t* q_empty = mma_done + 1;  // [2] Q_t free: every S_t product of an item completed
  uint64_t* o_empty = q_empty + 2;   // [2] O_t read out by the softmax warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int halo_tiles = a.halo / kPfTile;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_half[t], 4);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_final[t], 1);
      mbar_init(&o_empty[t], 4);
      mbar_init(&q_full[t], 1);
      mbar_init(&q_empty[t], 1);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Register split (whole warpgroups, each at one instruction address heading all of its
  // role code): launch 384 x 168 = 64512; after: 128 x 128 + 256 x 184 = 63488, and per SM
  // sub-partition (one warp of each group) 128 + 2 x 184 = 496 <= 512 registers per lane.
  if (warp < 4) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kPfRegsCtl));
  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      int kv_i = 0;             // running K/V tile counter
      int q_loads[2] = {0, 0};  // running Q_t loads
      bool ok = true;
      for (int w = blockIdx.x; ok && w < a.n_items; w += gridDim.x) {
        const PfItem I = pf_item(a, w);
        if (!I.act[0] && !I.act[1]) continue;
        // Q_t: after every S_t product of the previous item completed (Q_0 frees a step
        // before Q_1, so it loads while the previous item finishes)
        for (int t = 0; t < 2 && ok; ++t) {
          if (!I.act[t]) continue;
          if (q_loads[t] > 0 && !mbar_wait_bounded(&q_empty[t], (q_loads[t] - 1) & 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&q_full[t], L::kTileBytes);
          for (int bx = 0; bx < L::kBoxes; ++bx)
            tma_load_3d(smem + (t ? L::kQ1 : L::kQ0) + bx * L::kBoxBytes, &qmap, &q_full[t], bx * 64,
                        (I.qt0 + t) * kPfTile, I.bh);
          ++q_loads[t];
        }
        // K(j) before V(j): stages free in the order K(j-2) (after S(j-2)), V(j-2) (after PV(j-2))
        for (int j = I.J0; j <= I.J1; ++j) {
          const int i = kv_i++, s = i % kPfStages;
          const bool from_halo = j < halo_tiles;
          const CUtensorMap* km = from_halo ? &khmap : &kmap;
          const CUtensorMap* vm = from_halo ? &vhmap : &vmap;
          const int y = from_halo ? j * kPfTile : (j - halo_tiles) * kPfTile;
          if (i >= kPfStages && !mbar_wait_bounded(&k_empty[s], ((i / kPfStages) - 1) & 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[s], L::kTileBytes);
          for (int bx = 0; bx < L::kBoxes; ++bx)
            tma_load_3d(smem + L::kK + s * L::kTileBytes + bx * L::kBoxBytes, km, &k_full[s], bx * 64, y, I.bh);
          if (i >= kPfStages && !mbar_wait_bounded(&v_empty[s], ((i / kPfStages) - 1) & 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&v_full[s], L::kTileBytes);
          for (int bx = 0; bx < L::kBoxes; ++bx)
            tma_load_3d(smem + L::kV + s * L::kTileBytes + bx * L::kBoxBytes, vm, &v_full[s], bx * 64, y, I.bh);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    // The whole warp runs the control flow, so descriptors stay warp-uniform; one
    // elected lane (always the same one) issues each batch of tcgen05.mma and the
    // commits that track them.  Issuing from a single-lane branch instead costs about
    // twice the 64 cycles a 128x128x16 product takes on the tensor cores.
    constexpr uint32_t kIdQK = instr_desc_f16(PfFmt<T>::kFmt, kPfTile, kPfTile, 0, 0);
    constexpr uint32_t kIdPV = instr_desc_f16(PfFmt<T>::kFmt, kPfTile, D, 0, 1);
    // descriptor start addresses are in 16-byte units in the low 14 bits; smem offsets
    // below 256 KB never carry out of that field
    const uint64_t q_desc[2] = {smem_desc(smem_u32(smem + L::kQ0), 16, 1024),
                                smem_desc(smem_u32(smem + L::kQ1), 16, 1024)};
    const uint64_t k_desc = smem_desc(smem_u32(smem + L::kK), 16, 1024);
    const uint64_t v_desc = smem_desc(smem_u32(smem + L::kV), L::kBoxBytes, 1024);
    const uint32_t s_col[2] = {0u, 128u}, o_col[2] = {256u, 384u};
    auto commit = [&](uint64_t* bar) {
      if (elect_one_sync()) tc_commit(bar);
      __syncwarp();
    };
    // running counters: K/V tiles before this item, P signals per tile, items per tile
    int kv_base = 0;
    int it[2] = {0, 0}, o_uses[2] = {0, 0};
    bool ok = true;
    for (int w = blockIdx.x; ok && w < a.n_items; w += gridDim.x) {
      const PfItem I = pf_item(a, w);
      if (!I.act[0] && !I.act[1]) continue;
      const int J0 = I.J0, J1 = I.J1;
      bool q_ready[2] = {false, false};
      auto stage_of = [&](int j) { return (kv_base + j - J0) % kPfStages; };
      int k_ready = J0 - 1, v_ready = J0 - 1;  // last key tile whose K / V has been waited on
      auto wait_tile = [&](uint64_t* full, int& ready, int j) -> bool {
        if (j <= ready) return true;
        const int i = kv_base + j - J0;
        if (!mbar_wait_bounded(&full[i % kPfStages], (i / kPfStages) & 1)) return false;
        ready = j;
        tc_fence_after();
        return true;
      };
      // S_t = Q_t K(j)^T; the last one of the item frees Q_t for the next item
      auto issue_s = [&](int t, int j) -> bool {
        if (!q_ready[t]) {
          if (!mbar_wait_bounded(&q_full[t], o_uses[t] & 1)) return false;
          tc_fence_after();
          q_ready[t] = true;
        }
        const uint64_t kd = k_desc + ((stage_of(j) * L::kTileBytes) >> 4);
        if (elect_one_sync()) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = ((kk >> 2) * L::kBoxBytes + (kk & 3) * 32) >> 4;
            mma_ss(tmem + s_col[t], q_desc[t] + off, kd + off, kIdQK, kk > 0 ? 1u : 0u);
          }
          tc_commit(&s_full[t]);
          if (j == I.hi[t]) tc_commit(&q_empty[t]);
        }
        __syncwarp();
        return true;
      };
      // O_t += P_t V over key rows [16*k0, 16*k1) of the tile (P columns 8*k0 ..)
      auto issue_pv = [&](int t, uint64_t vd, int k0, int k1, bool first) {
        if (elect_one_sync()) {
#pragma unroll
          for (int kk = k0; kk < k1; ++kk)
            mma_ts(tmem + o_col[t], tmem + s_col[t] + kk * 8, vd + ((kk * 16 * 128) >> 4), kIdPV,
                   (!first || kk > 0) ? 1u : 0u);
        }
        __syncwarp();
      };
      // prologue: S_t(J0)
      if (ok && wait_tile(k_full, k_ready, J0)) {
        for (int t = 0; t < 2 && ok; ++t)
          if (I.act[t] && I.lo[t] <= J0 && J0 <= I.hi[t]) ok = issue_s(t, J0);
        commit(&k_empty[stage_of(J0)]);
      } else {
        ok = false;
      }
      for (int j = J0; ok && j <= J1; ++j) {
        const uint64_t vd = v_desc + ((stage_of(j) * L::kTileBytes) >> 4);
        for (int t = 0; t < 2 && ok; ++t) {
          if (I.act[t] && I.lo[t] <= j && j <= I.hi[t]) {
            const bool first = j == I.lo[t];
            // the first product of an item overwrites O_t: the previous item's O_t must
            // have been read out
            if (first && o_uses[t] > 0 && !mbar_wait_bounded(&o_empty[t], (o_uses[t] - 1) & 1)) {
              ok = false;
              break;
            }
            if (!mbar_wait_bounded(&p_half[t], it[t] & 1) || !wait_tile(v_full, v_ready, j)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(t, vd, 0, kPfTile / 32, first);
            if (!mbar_wait_bounded(&p_full[t], it[t] & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(t, vd, kPfTile / 32, kPfTile / 16, false);
            ++it[t];
            if (j == I.hi[t]) commit(&o_final[t]);
          }
          if (I.act[t] && I.lo[t] <= j + 1 && j + 1 <= I.hi[t]) {
            if (!wait_tile(k_full, k_ready, j + 1) || !issue_s(t, j + 1)) {
              ok = false;
              break;
            }
          }
        }
        // V(j) is free after PV(j); K(j+1) after both S(j+1) (the key-tile ranges of the two
        // query tiles overlap, so every j+1 <= J1 was used by at least one of them)
        commit(&v_empty[stage_of(j)]);
        if (ok && j + 1 <= J1) commit(&k_empty[stage_of(j + 1)]);
      }
      if (!ok) break;
#pragma unroll
      for (int t = 0; t < 2; ++t)
        if (I.act[t]) ++o_uses[t];
      kv_base += J1 - J0 + 1;
    }
    // every issued MMA completes before TMEM is released
    commit(mma_done);
    mbar_wait_bounded(mma_done, 0);
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kPfRegsSoftmax));
    // ---------------------------------------------------------------- softmax
    // warps 4-7: query tile 0, warps 8-11: query tile 1; thread = row = TMEM lane
    const int t = (warp - 4) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t s_addr = lane_base + (t ? 128u : 0u);
    const uint32_t o_addr = lane_base + (t ? 384u : 256u);
    unsigned char* stg = smem + L::kStage + (warp - 4) * 32 * L::kStageRow;
    int its = 0, o_cnt = 0;  // running: S signals of tile t, items with tile t
    bool ok = true;
    for (int w = blockIdx.x; ok && w < a.n_items; w += gridDim.x) {
      const PfItem I = pf_item(a, w);
      if (!I.act[t]) continue;
      const int qt = I.qt0 + t;
      const int qc = qt * kPfTile + r + a.halo;  // this row's query position
      const int tile_q0 = qt * kPfTile + a.halo;
      float m_run = -INFINITY, l_run = 0.f;
      int itl = 0;
      for (int j = I.lo[t]; j <= I.hi[t]; ++j) {
        if (!mbar_wait_bounded(&s_full[t], its & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int kc0 = j * kPfTile;
        const bool full_tile =
            kc0 + kPfTile - 1 <= tile_q0 && kc0 > tile_q0 + kPfTile - 1 - a.W && kc0 + kPfTile <= a.halo + a.S;
        // the whole row of S_t in registers: one TMEM round trip
        uint32_t sv[kPfTile];
        SPA_TMEM_LD32(s_addr, sv);
        SPA_TMEM_LD32(s_addr + 32, (sv + 32));
        SPA_TMEM_LD32(s_addr + 64, (sv + 64));
        SPA_TMEM_LD32(s_addr + 96, (sv + 96));
        tmem_wait_ld();
        if (!full_tile) {
          // scores outside [kmin, kmax] (causal, window, sequence end) become -inf; a row
          // with no key of this tile in range keeps none
          const int kmin = max(qc - a.W + 1 - kc0, 0);
          const int kmax = min(min(qc, a.halo + a.S - 1) - kc0, kPfTile - 1);
          const uint32_t span = kmax >= kmin ? static_cast<uint32_t>(kmax - kmin) : 0u;
          const int first = kmax >= kmin ? kmin : kPfTile;
#pragma unroll
          for (int e = 0; e < kPfTile; ++e)
            sv[e] = static_cast<uint32_t>(e - first) <= span ? sv[e] : 0xff800000u;
        }
        float mx[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) mx[c] = fmaxf(__uint_as_float(sv[2 * c]), __uint_as_float(sv[2 * c + 1]));
#pragma unroll
        for (int e = 16; e < kPfTile; e += 16) {
#pragma unroll
          for (int c = 0; c < 8; ++c)
            mx[c] = fmax3(mx[c], __uint_as_float(sv[e + 2 * c]), __uint_as_float(sv[e + 2 * c + 1]));
        }
        const float mt =
            fmaxf(fmax3(mx[0], mx[1], mx[2]), fmax3(fmax3(mx[3], mx[4], mx[5]), mx[6], mx[7])) * a.scale_log2;
        if (mt > m_run + kPfRescaleThreshold || (m_run == -INFINITY && mt > -INFINITY)) {
          // move the running max; rescale O (complete: S_t(j) was issued after O_t(j-1))
          const float alpha = fast_exp2(m_run - mt);  // 0 when m_run = -inf
          if (itl > 0 && m_run > -INFINITY) {
#pragma unroll 1
            for (int c = 0; c < D / 16; ++c) {
              uint32_t o[16];
              SPA_TMEM_LD16(o_addr + 16 * c, o);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
              SPA_TMEM_ST16(o_addr + 16 * c, o);
            }
          }
          l_run *= alpha;
          m_run = mt;
        }
        const float neg_mu = m_run == -INFINITY ? 0.f : -m_run;
        const float sc = a.scale_log2;
        // P = exp2(s*scale - m) as 16-bit pairs into columns [0, 64) of S_t: keys 0-63 into
        // [0, 32), signal, then keys 64-127 into [32, 64)
        const float2 sc2 = make_float2(sc, sc), nm2 = make_float2(neg_mu, neg_mu);
        float2 ls[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t pk[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float2 x = ffma2(
                make_float2(__uint_as_float(sv[64 * h + 2 * e]), __uint_as_float(sv[64 * h + 2 * e + 1])), sc2, nm2);
            const float2 pr = make_float2(fast_exp2(x.x), fast_exp2(x.y));
            ls[e & 1] = fadd2(ls[e & 1], pr);
            pk[e] = PfFmt<T>::pack(pr.x, pr.y);
          }
          SPA_TMEM_ST32(s_addr + 32 * h, pk);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(h == 0 ? &p_half[t] : &p_full[t]);
        }
        l_run += (ls[0].x + ls[0].y) + (ls[1].x + ls[1].y);
        ++its;
        ++itl;
      }
      if (!ok) break;
      // epilogue: O / l -> global through the warp's staging tile
      if (!mbar_wait_bounded(&o_final[t], o_cnt & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      const int q_row0 = qt * kPfTile + quad * 32;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        SPA_TMEM_LD32(o_addr + 32 * c, o);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          pk[e] = PfFmt<T>::pack(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
        uint4* mine = reinterpret_cast<uint4*>(stg + lane * L::kStageRow);
#pragma unroll
        for (int v = 0; v < 4; ++v) mine[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int row = k * 8 + (lane >> 2), part = lane & 3;
          const int qr = q_row0 + row;
          const uint4 v = *reinterpret_cast<const uint4*>(stg + row * L::kStageRow + part * 16);
          if (qr < a.row1)
            *reinterpret_cast<uint4*>(static_cast<T*>(a.out) + (static_cast<int64_t>(I.bh) * a.S + qr) * D + 32 * c +
                                      part * 8) = v;
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[t]);
      ++o_cnt;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

inline bool prefill_sm100_supported(const PrefillArgs& a, int dtype) {
  if (dtype != SPA_BF16 && dtype != SPA_F16) return false;
  if (a.D != 128 && a.D != 64) return false;
  if (a.halo % kPfTile != 0 || a.row0 % kPfTile != 0) return false;
  const uintptr_t m = reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
                      reinterpret_cast<uintptr_t>(a.v) | reinterpret_cast<uintptr_t>(a.out) |
                      reinterpret_cast<uintptr_t>(a.k_halo) | reinterpret_cast<uintptr_t>(a.v_halo);
  return (m & 15) == 0;
}

// SMs the persistent prefill grid leaves free (process-wide).
inline int& prefill_sm_reserve() {
  static int n = 0;
  return n;
}

template <typename T>
int launch_prefill_sm100(const PrefillArgs& a, int dtype, cudaStream_t st) {
  CUtensorMap qm, km, vm, khm, vhm;
  const uint64_t bh = static_cast<uint64_t>(a.B) * a.H;
  if (!spa_make_tensor_map_3d(&qm, a.q, dtype, a.D, a.S, bh) || !spa_make_tensor_map_3d(&km, a.k, dtype, a.D, a.S, bh) ||
      !spa_make_tensor_map_3d(&vm, a.v, dtype, a.D, a.S, bh))
    return SPA_ERR_INVALID;
  if (a.halo > 0) {
    if (!spa_make_tensor_map_3d(&khm, a.k_halo, dtype, a.D, a.halo, bh) ||
        !spa_make_tensor_map_3d(&vhm, a.v_halo, dtype, a.D, a.halo, bh))
      return SPA_ERR_INVALID;
  } else {
    khm = km;
    vhm = vm;
  }
  PfTcArgs t;
  t.out = a.out;
  t.S = a.S;
  t.W = a.W;
  t.halo = a.halo;
  t.row0 = a.row0;
  t.row1 = a.row1;
  t.H = a.H;
  const int tiles = (a.row1 - 1) / kPfTile - a.row0 / kPfTile + 1;
  t.n_pairs = (tiles + 1) / 2;
  const int64_t items = static_cast<int64_t>(t.n_pairs) * static_cast<int64_t>(bh);
  if (items > 0x7fffffff) return SPA_ERR_UNSUPPORTED;
  t.n_items = static_cast<int>(items);
  // persistent: one CTA per SM (the kernel's shared memory and TMEM admit one), minus the
  // SMs left to a concurrent halo exchange (spa_set_prefill_sm_reserve)
  const int sms = std::max(1, device_sm_count() - prefill_sm_reserve());
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(items, sms));
  t.scale_log2 = a.scale * 1.4426950408889634f;
  if (a.D == 128) {
    auto kern = prefill_tc_kernel<T, 128>;
    SPA_CHECK_CUDA(spa_set_smem_once(kern, PfSmem<128>::kBytes));
    kern<<<grid, kPfThreads, PfSmem<128>::kBytes, st>>>(qm, km, vm, khm, vhm, t);
  } else {
    auto kern = prefill_tc_kernel<T, 64>;
    SPA_CHECK_CUDA(spa_set_smem_once(kern, PfSmem<64>::kBytes));
    kern<<<grid, kPfThreads, PfSmem<64>::kBytes, st>>>(qm, km, vm, khm, vhm, t);
  }
  SPA_CHECK_CUDA(cudaGetLastError());
  return SPA_OK;
}

}  // namespace spa

extern "C" int spa_set_prefill_sm_reserve(int n) {
  const int prev = spa::prefill_sm_reserve();
  if (n >= 0) spa::prefill_sm_reserve() = n;
  return prev;
}
