// ql_prefill_tc.cu -- causal GQA flash-attention prefill on the 5th-gen tensor
// cores (tcgen05 + TMEM) for B200 (sm_100a).
//
// Replaces, for multi-token calls, the reference's per-head loop over the new
// rows (src/transformer/layers.rs:430-445: q_h.k_h^T, scale, offset causal
// mask :509-531, softmax ops.rs:292-319, probabilities.v_h).
//
// One CTA = 128 query rows of NQ query heads (two heads of one KV group when
// the group size is even) of one sequence; the heads share every K/V tile.
// Warp roles:
//   warp 0      TMA producer: the rotated Q tiles once, then K/V tiles of 128
//               keys (two 64-position page boxes x two 64-column halves each)
//               into a two-stage ring with separate K and V barriers; boxes of
//               unallocated pages are read out of range, which TMA fills with
//               zeros.
//   warp 1      owns TMEM (512 columns) and issues every tcgen05.mma from one
//               thread: S_q(j) = Q_q K_j^T (A and B from shared memory) and
//               O_q += P_q(j) V_j with P taken from TMEM; completion is
//               signalled with tcgen05.commit on mbarriers.  The two heads'
//               MMAs interleave, so one head's MMAs run while the other
//               head's softmax warpgroup works.
//   warps 2-3   bf16 caches only: convert each landed K/V tile to f16 in
//               shared memory, scaled per tile by a power of two into f16's
//               range (the MMAs wait for the converted tile).
//   warps 4..   one softmax warpgroup per head, one thread per query row (=
//               TMEM lane): read S (two passes of 32 columns: max, then
//               exp2), write P as f16 pairs over S's first 64 columns; keep a
//               running max that moves only when it grows by more than 2^8,
//               rescaling that row of O in TMEM then; finally normalise O and
//               store the output row.
// Operands are f16: the cache's f16 values, or its bf16 values times the
// tile's power of two (exact for every value that f16 can hold at that
// scale); q rotated in f32, divided by its row's power of two (1 unless the
// row reaches 2^15) and rounded to f16.  Each power of two is folded back
// into the scores or the output, so a bf16 cache keeps bf16's range.  The
// accumulators are f32 in TMEM.  No cluster multicast is used anywhere.
#include <math_constants.h>

#include <atomic>
#include <type_traits>

#include "ql_append.cuh"
#include "ql_device.cuh"
#include "ql_kernels.cuh"

namespace ql {

namespace {

constexpr int kBM = 128;  // query rows per CTA
constexpr int kBN = 128;  // keys per KV tile
constexpr float kLog2eP = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.f;  // rescale O only when the max grows by more than 2^8

// ------------------------------------------------------------ tcgen05 PTX --
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// D[tmem] (+)= A[smem] * B[smem], kind::f16, f32 accumulate.
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}
// 32 consecutive columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout code 2), sm100
// descriptor version 1.  lbo/sbo in bytes.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFF) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::f16 with f16 A/B and f32 D.
__host__ __device__ constexpr uint32_t instr_desc(int m, int n, bool b_mn_major) {
  return (1u << 4) | (b_mn_major ? (1u << 16) : 0u) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

// D[tmem] (+)= A[tmem] * B[smem], kind::f16 (A K-major in TMEM, two f16 per column).
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}
// 16 consecutive 32-bit columns of this thread's lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
// Register rebalancing between warpgroups.  The block launches with
// kThreads x 168 registers; the TMA/MMA warpgroup gives back down to 64 and
// each softmax warpgroup takes up to 216: 128*64 + 256*216 = 63488 <= 64512.
template <uint32_t N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ float ex2_approx(float x) {  // 2^x; -inf -> +0
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// NQ query tiles (heads 2p, 2p+1 of one KV group when NQ == 2) share every
// K/V tile.  TMEM columns: two S slots at [0, 128) and [128, 256), each with
// its P (f16 pairs) written over its first 64 columns, and O_q at
// [256 + 128q, 256 + 128q + HD).  Two heads: slot q holds head q's S.  One
// head: the slots alternate between KV tiles (S(j) in slot j & 1), so the
// next tile's S is computed while the softmax works on this one.
template <int HD, int NQ>
struct PrefillCfg {
  static constexpr int kHalves = HD / 64;
  static constexpr int kQBytes = kBM * HD * 2;     // per query tile: [half][128 rows][128 B]
  static constexpr int kKBytes = kBN * HD * 2;     // [half][128 keys][128 B]
  static constexpr int kStageBytes = 2 * kKBytes;  // K then V
  static constexpr int kStages = 2;
  static constexpr int kQOff = 0;
  static constexpr int kStageOff = kQOff + NQ * kQBytes;
  static constexpr int kBarOff = kStageOff + kStages * kStageBytes;
  static constexpr size_t kSmem = 1024 + kBarOff + 256;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kOCol = 256;
  static constexpr int kThreads = 128 * (1 + NQ);  // warpgroup 0: TMA + MMA; one per tile
};

}  // namespace

template <int HD, int NQ, bool BF>
__global__ void __launch_bounds__(PrefillCfg<HD, NQ>::kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ PrefillArgs a, const __grid_constant__ CUtensorMap qmap,
                      const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap) {
  using C = PrefillCfg<HD, NQ>;
  const int n_qt = (a.new_len + kBM - 1) / kBM;
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.x);  // heaviest tiles first
  const int h0 = blockIdx.y * NQ, b = blockIdx.z;
  const int kvh = h0 / a.group;
  const int seq = a.seqs.seq[b];
  const int start = a.seqs.start[b];
  const int q_first = qt * kBM;
  const int q_last = min(a.new_len, q_first + kBM) - 1;
  const int kv_end = start + q_last + 1;  // keys visible to the last row
  const int n_kv = (kv_end + kBN - 1) / kBN;
  const int hkv = a.cache.hkv;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* qsm = smem + C::kQOff;
  uint8_t* stg = smem + C::kStageOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* q_full = bars + 0;
  // K and V of a tile have their own barriers: K is free once the tile's
  // last S MMA is done, V only after its last PV, so K's refill starts about
  // an iteration earlier than a shared K/V stage would allow.
  uint64_t* k_full = bars + 11;   // [2]
  uint64_t* k_empty = bars + 13;  // [2]
  uint64_t* v_full = bars + 15;   // [2]
  uint64_t* v_empty = bars + 17;  // [2]
  // One head per CTA (DB): the two S slots alternate between KV tiles, so
  // s_full/p_full are per slot and the softmax waits for P(j-1).V through
  // o_full before it rescales O.  Two heads: slot = head.
  constexpr bool DB = NQ == 1;
  uint64_t* s_full = bars + 5;    // [2] S of the slot computed (and everything issued before it)
  uint64_t* p_full = bars + 7;    // [2] P of the slot written, O rescaled if needed
  uint64_t* o_done = bars + 9;    // all MMAs complete
  uint64_t* o_full = bars + 19;   // DB: P(j).V complete, one phase per KV tile but the last
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int q = 0; q < 2; ++q) {
      mbar_init(&s_full[q], 1);
      mbar_init(&p_full[q], 128);
    }
    mbar_init(o_done, 1);
    mbar_init(o_full, 1);
    fence_mbar_init();
    tma_prefetch_desc(&qmap);
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();

  if (warp < 4) {
  if constexpr (NQ == 2) regs_dec<64>();
  if (warp == 0) {
    // -------------------------------------------------------- producer --
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, NQ * C::kQBytes);
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        const int qrow = (b * a.hq + h0 + q) * a.q_rows + q_first;
#pragma unroll
        for (int hf = 0; hf < C::kHalves; ++hf)
          tma_load_2d(qsm + q * C::kQBytes + hf * (kBM * 128), &qmap, hf * 64, qrow, q_full);
      }
    }
    // Page rows of 32 sub-tiles (64 keys each) at a time, one per lane, so no
    // dependent global load sits between two copies; lane 0 issues the K/V
    // tiles of 128 keys as stages free up.
    const int* bt = a.cache.block_table + static_cast<size_t>(seq) * a.cache.pages_per_seq;
    const int oob_row = a.cache.num_pages * hkv * a.cache.page;  // past the pool: zero fill
    bool alive = true;
    for (int c0 = 0; c0 < 2 * n_kv && alive; c0 += 32) {
      const int u = c0 + lane, key0 = u * 64;
      int lane_row = oob_row;
      if (BF) {  // the dense f16 copy: rows of this (sequence, KV head) in key order
        lane_row = (b * hkv + kvh) * a.kv_rows + key0;
      } else if (u < 2 * n_kv && key0 / a.cache.page < a.cache.pages_per_seq) {
        const int page = __ldg(bt + key0 / a.cache.page);
        if (page >= 0 && page < a.cache.num_pages)
          lane_row = (page * hkv + kvh) * a.cache.page + key0 % a.cache.page;
      }
      const int n = min(32, 2 * n_kv - c0);
      for (int jj = 0; jj < n && alive; jj += 2) {
        const int rows[2] = {__shfl_sync(0xffffffffu, lane_row, jj),
                             __shfl_sync(0xffffffffu, lane_row, jj + 1)};
        if (lane == 0) {
          const int j = (c0 + jj) / 2, st = j & 1;
          uint8_t* ks = stg + st * C::kStageBytes;
          uint8_t* vs = ks + C::kKBytes;
          if (j >= 2 && !mbar_wait(&k_empty[st], ((j >> 1) - 1) & 1, a.status)) {
            alive = false;
          } else {
            mbar_arrive_expect_tx(&k_full[st], C::kKBytes);
#pragma unroll
            for (int sub = 0; sub < 2; ++sub)
#pragma unroll
              for (int hf = 0; hf < C::kHalves; ++hf)
                tma_load_2d(ks + hf * (kBN * 128) + sub * 8192, &kmap, hf * 64, rows[sub],
                            &k_full[st]);
          }
          if (alive && j >= 2 && !mbar_wait(&v_empty[st], ((j >> 1) - 1) & 1, a.status)) {
            alive = false;
          } else if (alive) {
            mbar_arrive_expect_tx(&v_full[st], C::kKBytes);
#pragma unroll
            for (int sub = 0; sub < 2; ++sub)
#pragma unroll
              for (int hf = 0; hf < C::kHalves; ++hf)
                tma_load_2d(vs + hf * (kBN * 128) + sub * 8192, &vmap, hf * 64, rows[sub],
                            &v_full[st]);
          }
        }
        alive = __shfl_sync(0xffffffffu, alive, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA --
    // Issue order per KV tile j (the tensor core executes them in order):
    //   PV_0(j-1) S_0(j) PV_1(j-1) S_1(j) ...   so that while one softmax
    //   warpgroup works on S_q(j), the other query tile's MMAs run.
    if (lane == 0) {
      constexpr uint32_t idesc_s = instr_desc(kBM, kBN, false);
      constexpr uint32_t idesc_o = instr_desc(kBM, HD, true);
      const uint32_t qaddr = smem_u32(qsm);
      bool ok = mbar_wait(q_full, 0, a.status);
      // slot: the S/P columns (head q, or tile parity with one head)
      auto issue_s = [&](int q, int slot, int j) {
        const uint32_t kaddr = smem_u32(stg + (j & 1) * C::kStageBytes);
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
          const uint32_t koff = (ks >> 2) * (kBN * 128) + (ks & 3) * 32;
          const uint32_t qoff = q * C::kQBytes + (ks >> 2) * (kBM * 128) + (ks & 3) * 32;
          tc_mma(tmem + slot * kBN, smem_desc(qaddr + qoff, 16, 1024),
                 smem_desc(kaddr + koff, 16, 1024), idesc_s, ks > 0);
        }
        tc_commit(&s_full[slot]);
      };
      auto issue_pv = [&](int q, int slot, int j) {
        const uint32_t vaddr = smem_u32(stg + (j & 1) * C::kStageBytes + C::kKBytes);
#pragma unroll
        for (int ks = 0; ks < kBN / 16; ++ks)
          tc_mma_ts(tmem + C::kOCol + q * 128, tmem + slot * kBN + ks * 8,
                    smem_desc(vaddr + ks * 2048, kBN * 128, 1024), idesc_o, (j > 0 || ks > 0));
      };
      if constexpr (DB) {
        // S(j) into slot j & 1 as soon as K(j) lands (the slot's P(j-2) was
        // read by P(j-2).V, issued before it), then P(j-1).V once the
        // softmax has written P(j-1): the tensor core runs S(j) while the
        // softmax works on S(j-1).
        for (int j = 0; ok && j < n_kv; ++j) {
          ok = mbar_wait(&k_full[j & 1], (j >> 1) & 1, a.status);
          if (!ok) break;
          tc_fence_after();
          issue_s(0, j & 1, j);
          tc_commit(&k_empty[j & 1]);
          if (j > 0) {
            ok = mbar_wait(&p_full[(j - 1) & 1], ((j - 1) >> 1) & 1, a.status) &&
                 mbar_wait(&v_full[(j - 1) & 1], ((j - 1) >> 1) & 1, a.status);
            if (!ok) break;
            tc_fence_after();
            issue_pv(0, (j - 1) & 1, j - 1);
            tc_commit(&v_empty[(j - 1) & 1]);
            tc_commit(o_full);
          }
        }
        const int last = n_kv - 1;
        if (ok) ok = mbar_wait(&p_full[last & 1], (last >> 1) & 1, a.status) &&
                     mbar_wait(&v_full[last & 1], (last >> 1) & 1, a.status);
        if (ok) {
          tc_fence_after();
          issue_pv(0, last & 1, last);
        }
      } else {
        for (int j = 0; ok && j < n_kv; ++j) {
          ok = mbar_wait(&k_full[j & 1], (j >> 1) & 1, a.status);
          if (ok && j > 0) ok = mbar_wait(&v_full[(j - 1) & 1], ((j - 1) >> 1) & 1, a.status);
          if (!ok) break;
          for (int q = 0; q < NQ; ++q) {
            if (j > 0) {  // P_q(j-1) is in S_q's columns: consume it before S_q(j) overwrites them
              if (!mbar_wait(&p_full[q], (j - 1) & 1, a.status)) {
                ok = false;
                break;
              }
              tc_fence_after();
              issue_pv(q, q, j - 1);
              if (q == NQ - 1) tc_commit(&v_empty[(j - 1) & 1]);
            }
            tc_fence_after();
            issue_s(q, q, j);
          }
          if (ok) tc_commit(&k_empty[j & 1]);  // every S of tile j reads K(j) only
        }
        if (ok) ok = mbar_wait(&v_full[(n_kv - 1) & 1], ((n_kv - 1) >> 1) & 1, a.status);
        for (int q = 0; ok && q < NQ; ++q) {
          if (!mbar_wait(&p_full[q], (n_kv - 1) & 1, a.status)) break;
          tc_fence_after();
          issue_pv(q, q, n_kv - 1);
        }
      }
      tc_commit(o_done);
    }
  }
  } else {
    if constexpr (NQ == 2) regs_inc<216>();
    // --------------------------------------------------------- softmax --
    const int q = (warp - 4) >> 2;     // which query tile this warpgroup serves
    const int r = threadIdx.x & 127;   // row in the tile == TMEM lane
    const int h = h0 + q;
    const int row = q_first + r;
    const int qpos = start + row;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t o_col = C::kOCol + q * 128;
    // The row's q was stored divided by its q_scale: the score scale puts it
    // back.  bf16 caches: tile j's K arrives divided by 2^k_exp[j] (folded
    // into that tile's score scale) and its V by 2^v_exp[j]; O accumulates
    // P.V / 2^ev_used, ev_used the largest V exponent so far, so tile j's P
    // is stored times 2^(v_exp[j] - ev_used) and O is rescaled when ev_used
    // grows (the sum l stays in unscaled P).
    const float sl2_row =
        a.scale * kLog2eP * a.q_scale[(static_cast<size_t>(b) * a.hq + h) * a.q_rows + row];
    int ev_used = -1000;  // set by the first tile
    // bf16: this (sequence, KV head)'s tile exponents, K then V
    const int8_t* tile_exp =
        BF ? a.tile_exp + (static_cast<size_t>(b) * hkv + kvh) * (a.kv_rows / kBN) : nullptr;
    const size_t v_exp_off = BF ? static_cast<size_t>(a.batch) * hkv * (a.kv_rows / kBN) : 0;
    float m_used = -CUDART_INF_F, l = 0.f;
    // tcgen05.ld/st are warp-collective (.sync.aligned): every branch around
    // them below is taken by whole warps, decided with warp votes.
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int slot = DB ? (j & 1) : q;
      const uint32_t s_col = slot * kBN;
      const uint32_t s_par = DB ? ((j >> 1) & 1) : (j & 1);
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[slot], s_par, a.status))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sl2 = sl2_row;
      if constexpr (BF) {
        const int ek = tile_exp[j];
        if (ek) sl2 *= pow2f(ek);
      }
      const int key0 = j * kBN;
      if (!BF && q == 0 && j == n_kv - 1 && key0 + r >= kv_end &&
          mbar_wait(&v_full[j & 1], (j >> 1) & 1, a.status)) {
        // Key r of the last tile lies past the sequence end: its V row may be
        // stale pool memory (Inf/NaN), and P = 0 times Inf would still reach
        // O.  Zero it once V has landed and before the PV MMAs read it (every
        // PV of this tile is issued after P_0 is released).
        uint8_t* vrow = stg + (j & 1) * C::kStageBytes + C::kKBytes + r * 128;
#pragma unroll
        for (int hf = 0; hf < C::kHalves; ++hf)
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(vrow + hf * (kBN * 128) + c * 16) = make_uint4(0, 0, 0, 0);
        fence_proxy_async_smem();
      }
      // The whole S row in registers: four loads, one wait.
      float x[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) {
        float v[32];
        tmem_ld32(lane_addr + s_col + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) x[c * 32 + i] = v[i];
      }
      tmem_wait_ld();
      if (key0 + kBN - 1 > qpos) {  // diagonal tile: keys after this row's position are masked
        const int lim = qpos - key0;  // keys 0..lim visible
#pragma unroll
        for (int i = 0; i < kBN; ++i)
          if (i > lim) x[i] = -CUDART_INF_F;
      }
      float m8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) m8[e] = x[e];
#pragma unroll
      for (int i = 8; i < kBN; ++i) m8[i & 7] = fmaxf(m8[i & 7], x[i]);
      float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                       fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
      mx = __fmul_rn(mx, sl2);
      float corr = 1.f;
      bool rescale = false;
      if (mx > m_used + kRescaleLog2 || m_used == -CUDART_INF_F) {
        const float m_new = mx == -CUDART_INF_F ? 0.f : mx;
        corr = ex2_approx(m_used - m_new);  // 0 while nothing has been accumulated
        rescale = j > 0 && m_used != -CUDART_INF_F;
        m_used = m_new;
      }
      // The warp rescales its O rows together; rows that kept their maximum
      // multiply by exactly 1.
      rescale = __any_sync(0xffffffffu, rescale);
      // p = 2^(s*scale*log2e - m), packed f16 pairs over S's first 64 columns.
      // m_used is the rounded product max(s)*scale*log2e; a fused multiply-add
      // against it is off by up to half an ulp of that product, harmless
      // below 2^20 but an overflow of 2^(...) for scores far above any
      // attention's usual range, where the rounded products are subtracted
      // instead (the largest then gives exactly 2^0).
      float ps[4] = {0.f, 0.f, 0.f, 0.f};
      auto emit_p = [&](auto exact) {
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            float p0, p1;
            if constexpr (decltype(exact)::value) {
              // __fmul_rn: the product must be rounded on its own, not
              // contracted into a multiply-add
              p0 = ex2_approx(__fmul_rn(x[c * 32 + i], sl2) - m_used);
              p1 = ex2_approx(__fmul_rn(x[c * 32 + i + 1], sl2) - m_used);
            } else {
              p0 = ex2_approx(fmaf(x[c * 32 + i], sl2, -m_used));
              p1 = ex2_approx(fmaf(x[c * 32 + i + 1], sl2, -m_used));
            }
            ps[(i >> 1) & 3] += p0 + p1;
            __half2 hp = __floats2half2_rn(p0, p1);
            pk[i >> 1] = *reinterpret_cast<uint32_t*>(&hp);
          }
          tmem_st16(lane_addr + s_col + c * 16, pk);
        }
      };
      if (__any_sync(0xffffffffu, fabsf(m_used) >= 1048576.f))
        emit_p(std::true_type{});
      else
        emit_p(std::false_type{});
      l = l * corr + ((ps[0] + ps[1]) + (ps[2] + ps[3]));
      float ocorr = corr;  // O's factor
      if constexpr (BF) {
        // P(j) went out for ev == ev_used: a larger ev rescales O instead, a
        // smaller one scales P(j) down (both rare: tiles of ordinary data all
        // have exponent 0).
        const int ev = tile_exp[v_exp_off + j];
        if (ev > ev_used) {
          if (j > 0) {
            ocorr *= pow2f(ev_used - ev);
            rescale = true;
          }
          ev_used = ev;
        } else if (ev < ev_used) {
          const float pf = pow2f(ev - ev_used);
          tmem_wait_st();
#pragma unroll
          for (int c = 0; c < kBN / 64; ++c) {
            float v[32];
            tmem_ld32(lane_addr + s_col + c * 32, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&v[i]));
              __half2 hp = __floats2half2_rn(f2.x * pf, f2.y * pf);
              v[i] = *reinterpret_cast<const float*>(&hp);
            }
            tmem_st32(lane_addr + s_col + c * 32, v);
          }
        }
      }
      if (DB && rescale) {  // O is final only once P(j-1).V has completed
        if (!__all_sync(0xffffffffu, mbar_wait(o_full, (j - 1) & 1, a.status))) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if (rescale) {  // two heads: the previous P_q.V is complete, S_q(j) was issued after it
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          float v[32];
          tmem_ld32(lane_addr + o_col + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= ocorr;
          tmem_st32(lane_addr + o_col + c * 32, v);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[slot]);
    }
    // ---- epilogue: O / l for the valid rows
    if (__all_sync(0xffffffffu, ok && mbar_wait(o_done, 0, a.status))) {
      tc_fence_after();
      const float inv = (BF ? pow2f(ev_used) : 1.f) / l;
      const size_t obase = ((static_cast<size_t>(b) * a.new_len + row) * a.hq + h) * HD;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        float v[32];
        tmem_ld32(lane_addr + o_col + c * 32, v);
        tmem_wait_ld();
        if (row < a.new_len) {
          if (a.out_dtype == kF32) {
            float4* o4 = reinterpret_cast<float4*>(static_cast<float*>(a.out) + obase + c * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              o4[i] = make_float4(v[4 * i] * inv, v[4 * i + 1] * inv, v[4 * i + 2] * inv,
                                  v[4 * i + 3] * inv);
          } else {
            uint4* o4 = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + obase + c * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t w4[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float x0 = v[8 * i + 2 * e] * inv, x1 = v[8 * i + 2 * e + 1] * inv;
                w4[e] = a.out_dtype == kF16 ? pack2<false>(x0, x1) : pack2<true>(x0, x1);
              }
              o4[i] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
            }
          }
        }
      }
    }
  }
  griddep_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// Query heads per prologue warp: the position's (cos, sin) pairs are read
// once and serve every head of the group.
constexpr int kQHeads = 4;

// The rotated q rows of one (sequence, query row t, group of kQHeads heads),
// warp-wide; padding rows of the last 128-row tile (t >= new_len) are written
// as zeros, never left as stale memory.  Each lane moves HD/32 consecutive
// values of a row.  A row is stored divided by 2^e, e = f16_range_exp of its
// largest magnitude (0 for ordinary data, leaving the f16 rounding as it
// was), and 2^e goes to q_scale for the attention kernel to fold into the
// row's score scale.
template <int HD>
__device__ __forceinline__ void prologue_q(const PrefillArgs& a, int w, int lane) {
  constexpr int kN = HD / 32;
  const int ng = (a.hq + kQHeads - 1) / kQHeads;
  const int g = w % ng, bt = w / ng;
  const int t = bt % a.q_rows, b = bt / a.q_rows;
  const int h0 = g * kQHeads, h1 = min(a.hq, h0 + kQHeads);
  if (t >= a.new_len) {
    for (int h = h0; h < h1; ++h) {
      const size_t qrow = (static_cast<size_t>(b) * a.hq + h) * a.q_rows + t;
      const float z[kN] = {};
      store_vec<kN>(a.q_rot, qrow * HD + kN * lane, kF16, z);
      if (lane == 0) a.q_scale[qrow] = 1.f;
    }
    return;
  }
  const int pos = a.seqs.start[b] + t;
  double2 cs[kN / 2];
#pragma unroll
  for (int i = 0; i < kN / 2; ++i)
    cs[i] = a.rope[static_cast<size_t>(pos) * a.rope_stride + lane * (kN / 2) + i];
  const bool vec =
      reinterpret_cast<uintptr_t>(a.q) % (static_cast<uintptr_t>(kN) * (a.in_dtype == kF32 ? 4 : 2)) == 0;
  // every head's row first: one memory round trip for the group, not one per head
  float ys[kQHeads][kN];
#pragma unroll
  for (int hh = 0; hh < kQHeads; ++hh) {
    if (h0 + hh < h1)
      load_vec<kN>(a.q, (static_cast<size_t>(b * a.new_len + t) * a.hq + h0 + hh) * HD + kN * lane,
                   a.in_dtype, vec, ys[hh]);
  }
#pragma unroll
  for (int hh = 0; hh < kQHeads; ++hh) {
    const int h = h0 + hh;
    if (h >= h1) break;
    float* y = ys[hh];
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < kN / 2; ++i) {
      rope_pair(y[2 * i], y[2 * i + 1], cs[i], y[2 * i], y[2 * i + 1]);
      m = fmaxf(m, fmaxf(fabsf(y[2 * i]), fabsf(y[2 * i + 1])));
    }
    const int e = f16_range_exp(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
    const float f = pow2f(-e);
    float yo[kN];
#pragma unroll
    for (int i = 0; i < kN; ++i) yo[i] = y[i] * f;
    const size_t qrow = (static_cast<size_t>(b) * a.hq + h) * a.q_rows + t;
    store_vec<kN>(a.q_rot, qrow * HD + kN * lane, kF16, yo);
    if (lane == 0) a.q_scale[qrow] = pow2f(e);
  }
}

// Warp w of the prologue grid: first the q groups, then (fused calls) one
// new token's K/V rows for every KV head.
template <int HD>
__device__ __forceinline__ void prologue_warp(const PrefillArgs& a, const AppendArgs& ap, int w,
                                              int lane) {
  const int q_warps = a.batch * a.q_rows * ((a.hq + kQHeads - 1) / kQHeads);
  if (w < q_warps) {
    prologue_q<HD>(a, w, lane);
    return;
  }
  const int r = w - q_warps;
  if (r < ap.batch * ap.new_len) append_token<HD>(ap, r, lane);
}

// -------------------------------------------------------------- prologue --
// One launch before the attention kernel, one warp per (sequence, query row,
// group of query heads), then, when the call's append is fused in, one warp
// per new token: K rotated with the host table (bit for bit the reference's
// rotation), K and V converted and written into the cache (the append of
// layers.rs:397-413 / cache.rs:146-163); rotated q lands at
// q_rot[((b*hq + h)*q_rows + t)*hd + d].
// Launched with programmatic dependent launch: everything it reads or writes
// comes after the grid dependency wait.  Each block lets the attention kernel
// launch only once its own rows are written: an attention CTA holds most of an
// SM's registers while it waits, so releasing it early would starve the
// prologue's remaining blocks; released at the end, its set-up (barriers,
// TMEM, descriptors) overlaps the prologue's last wave.
__global__ void __launch_bounds__(128) prefill_prologue_kernel(const __grid_constant__ PrefillArgs a,
                                                               const __grid_constant__ AppendArgs ap) {
  const int w = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  griddep_wait();
  if (a.cache.hd == 64)
    prologue_warp<64>(a, ap, w, lane);
  else
    prologue_warp<128>(a, ap, w, lane);
  griddep_launch_dependents();
}

// ------------------------------------------------- f16 copy of the keys --
// bf16 and Q8_0 caches: one CTA per (128-key tile, K or V, KV head,
// sequence) copies the keys the call sees into the dense f16 scratch, two
// threads per key row (each HD/2 values: bf16 as stored, Q8_0 dequantised
// exactly in f32, int8 times its block's f16 scale).  The tile is divided by
// 2^e, e = f16_range_exp of its largest magnitude (0 for ordinary data;
// otherwise the power of two that puts the tile into [2^14, 2^15)), and e goes
// to tile_exp for the attention kernel to fold back.  bf16 values convert
// exactly at that scale, apart from magnitudes under 2^(e-24); dequantised
// Q8_0 values (up to 19 significant bits) round to f16's 11.  Keys past the
// sequence's end (and rows of unallocated pages) are zeros.  Converting once
// here, instead of in every attention CTA that reads the tile, costs one read
// and one write of the keys (a few per cent of a long prefill) and keeps the
// attention kernel's pipeline that of an f16 cache.
template <int HD, int DT>
__global__ void __launch_bounds__(256) tiles_to_f16_kernel(const __grid_constant__ PrefillArgs a) {
  static_assert(DT == kBF16 || DT == kQ8_0, "bf16 or Q8_0 storage");
  constexpr int kVals = HD / 2;    // values per thread
  constexpr int kPer = kVals / 8;  // 8-value groups per thread
  const int tile = blockIdx.x, kind = blockIdx.y & 1, kvh = blockIdx.y >> 1, b = blockIdx.z;
  const int hkv = a.cache.hkv;
  const int kv_end = a.seqs.start[b] + a.new_len;
  if (tile * kBN >= kv_end) return;  // never read
  const int key = tile * kBN + (threadIdx.x >> 1), part = threadIdx.x & 1;
  griddep_wait();
  float v[kVals];
  bool live = key < kv_end;
  size_t row = 0;
  if (live) {
    const int page = a.cache.block_table[static_cast<size_t>(a.seqs.seq[b]) * a.cache.pages_per_seq +
                                         key / a.cache.page];
    live = page >= 0 && page < a.cache.num_pages;
    row = (static_cast<size_t>(page) * hkv + kvh) * a.cache.page + key % a.cache.page;
  }
  if (!live) {
#pragma unroll
    for (int i = 0; i < kVals; ++i) v[i] = 0.f;
  } else if constexpr (DT == kBF16) {
    const uint4* src = reinterpret_cast<const uint4*>(
        static_cast<const uint16_t*>(kind ? a.cache.v : a.cache.k) + row * HD + part * kVals);
#pragma unroll
    for (int g = 0; g < kPer; ++g) {
      const uint4 w = src[g];
      const uint32_t in[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        v[8 * g + 2 * k] = __uint_as_float(in[k] << 16);
        v[8 * g + 2 * k + 1] = __uint_as_float(in[k] & 0xffff0000u);
      }
    }
  } else {
    const uint4* src = reinterpret_cast<const uint4*>(
        static_cast<const int8_t*>(kind ? a.cache.v : a.cache.k) + row * HD + part * kVals);
    const uint16_t* sc = (kind ? a.cache.v_scale : a.cache.k_scale) + row * (HD / 32) +
                         part * (kVals / 32);
#pragma unroll
    for (int q = 0; q < kVals / 16; ++q) {  // 16 int8 values per load
      const uint4 w = src[q];
      const float d = __half2float(__ushort_as_half(sc[q / 2]));  // 32-value blocks
      const uint32_t in[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int byte = 0; byte < 4; ++byte)
          v[16 * q + 4 * k + byte] =
              static_cast<float>(static_cast<int8_t>((in[k] >> (8 * byte)) & 0xffu)) * d;
    }
  }
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < kVals; ++i) m = fmaxf(m, fabsf(v[i]));
  __shared__ uint32_t wmax[8];
  const uint32_t mb = __reduce_max_sync(0xffffffffu, __float_as_uint(m));
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = mb;
  __syncthreads();
  uint32_t tb = wmax[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) tb = max(tb, wmax[i]);
  const int e = f16_range_exp(tb);
  const float f = pow2f(-e);
  const int kv_tiles = a.kv_rows / kBN;
  if (threadIdx.x == 0)
    a.tile_exp[((static_cast<size_t>(kind) * a.batch + b) * hkv + kvh) * kv_tiles + tile] =
        static_cast<int8_t>(e);
  uint4* dst = reinterpret_cast<uint4*>((kind ? a.v_copy : a.k_copy) +
                                        ((static_cast<size_t>(b) * hkv + kvh) * a.kv_rows + key) * HD +
                                        part * kVals);
#pragma unroll
  for (int g = 0; g < kPer; ++g) {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const __half2 h = __floats2half2_rn(v[8 * g + 2 * k] * f, v[8 * g + 2 * k + 1] * f);
      w[k] = *reinterpret_cast<const uint32_t*>(&h);
    }
    dst[g] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  griddep_launch_dependents();
}

bool prefill_tc_supported(int hd, int dtype, int new_len) {
  return (hd == 64 || hd == 128) && (dtype == kF16 || dtype == kBF16 || dtype == kQ8_0) &&
         new_len >= 64;
}

size_t prefill_q_rows(int new_len) { return static_cast<size_t>((new_len + kBM - 1) / kBM) * kBM; }

template <int HD, int NQ, bool BF>
static cudaError_t launch_prefill_nq(const PrefillArgs& a, const CUtensorMap* qmap,
                                     const CUtensorMap* kmap, const CUtensorMap* vmap,
                                     cudaStream_t s) {
  using C = PrefillCfg<HD, NQ>;
  constexpr int kMaxDev = 64;
  static std::atomic<bool> configured[kMaxDev];  // shared-memory limit set on that device
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= kMaxDev || !configured[dev].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(prefill_tc_kernel<HD, NQ, BF>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(C::kSmem));
    if (e != cudaSuccess) return e;
    if (dev < kMaxDev) configured[dev].store(true, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.new_len + kBM - 1) / kBM, a.hq / NQ, a.batch);
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, prefill_tc_kernel<HD, NQ, BF>, a, *qmap, *kmap, *vmap);
}

template <int HD, bool BF>
static cudaError_t launch_prefill_hd(const PrefillArgs& a, const CUtensorMap* qmap,
                                     const CUtensorMap* kmap, const CUtensorMap* vmap,
                                     cudaStream_t s) {
  // Two heads of one KV group per CTA (one head's MMAs run while the other's
  // softmax works) when the group has an even size and the grid still covers
  // the SMs; a small call takes one head per CTA for twice the CTAs.
  const long long tiles = (a.new_len + kBM - 1) / kBM;
  const long long pair_ctas = tiles * (a.hq / 2) * a.batch;
  if (a.group % 2 == 0 && pair_ctas >= a.num_sms)
    return launch_prefill_nq<HD, 2, BF>(a, qmap, kmap, vmap, s);
  return launch_prefill_nq<HD, 1, BF>(a, qmap, kmap, vmap, s);
}

cudaError_t launch_prefill_tc(const PrefillArgs& a, const AppendArgs& ap, const CUtensorMap* qmap,
                              const CUtensorMap* kmap, const CUtensorMap* vmap, cudaStream_t s) {
  const long long q_rows = static_cast<long long>(a.batch) * a.q_rows * ((a.hq + kQHeads - 1) / kQHeads);
  const long long kv_rows = static_cast<long long>(ap.batch) * ap.new_len;
  // A call of a few waves of attention CTAs is bound by launch latency: one
  // prologue launch with programmatic dependent launch.  A large one keeps the
  // append and the rotation as two ordinary launches (measured a few per cent
  // faster on 4 x 8192 tokens, where their traffic, not their latency, counts).
  const long long ctas = static_cast<long long>((a.new_len + kBM - 1) / kBM) * a.hq * a.batch;
  // (append_token writes f32/f16/bf16 rows; a Q8_0 cache appends through
  // append_kernel, which quantises its blocks)
  const bool fused = ctas < 8LL * a.num_sms && a.cache.dtype != kQ8_0;
  PrefillArgs qa = a;
  AppendArgs none = ap;
  none.new_len = 0;
  if (!fused && kv_rows > 0) {
    cudaError_t e = launch_append(ap, s);
    if (e != cudaSuccess) return e;
  }
  const long long rows = q_rows + (fused ? kv_rows : 0);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((rows + 3) / 4));
  cfg.blockDim = dim3(128);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = fused ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, prefill_prologue_kernel, qa, fused ? ap : none);
  if (e != cudaSuccess) return e;
  const bool bf = a.cache.dtype == kBF16 || a.cache.dtype == kQ8_0;  // reads the f16 copy
  if (bf) {  // the keys as f16 tiles, after the rows this call appends
    cudaLaunchConfig_t cc = {};
    cc.gridDim = dim3(static_cast<unsigned>(a.kv_rows / kBN), 2u * a.cache.hkv,
                      static_cast<unsigned>(a.batch));
    cc.blockDim = dim3(256);
    cc.stream = s;
    cc.attrs = attr;
    cc.numAttrs = 1;
    const bool q8 = a.cache.dtype == kQ8_0;
    if (a.cache.hd == 64)
      e = q8 ? cudaLaunchKernelEx(&cc, tiles_to_f16_kernel<64, kQ8_0>, a)
             : cudaLaunchKernelEx(&cc, tiles_to_f16_kernel<64, kBF16>, a);
    else
      e = q8 ? cudaLaunchKernelEx(&cc, tiles_to_f16_kernel<128, kQ8_0>, a)
             : cudaLaunchKernelEx(&cc, tiles_to_f16_kernel<128, kBF16>, a);
    if (e != cudaSuccess) return e;
  }
  if (a.cache.hd == 64)
    return bf ? launch_prefill_hd<64, true>(a, qmap, kmap, vmap, s)
              : launch_prefill_hd<64, false>(a, qmap, kmap, vmap, s);
  return bf ? launch_prefill_hd<128, true>(a, qmap, kmap, vmap, s)
            : launch_prefill_hd<128, false>(a, qmap, kmap, vmap, s);
}

}  // namespace ql
