// Dense GEMMs on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
//   C[M,N] = A[M,K] @ B[K,N]          (int8 -> int32, bf16 -> f32 / bf16)
//   C[M,N] = A[M,K] @ W[N,K]^T (+bias) (bf16 linear layer, W in nn.Linear layout)
//   C[M,N] = A[M,K] @ B[K,N]          (int16 -> int32 via int8 limb products)
//
// Reference: examples/matmul_i8_m128_n64_k64/matmul_i8_m128_n64_k64.py:22-52
// (`bare_matmul_i8`, i8 x i8 -> i32), examples/matmul_bf16_m64_n64_k64/
// matmul_bf16_m64_n64_k64.py:16-46 and examples/autotune-matmul/matmul.py:22-53
// (`bare_matmul`, bf16 x bf16 -> f32), examples/qwen2_5/kernels/matmul.py:172-296
// (`triton_linear`, x @ W^T + b).  The reference's i8/i16 accumulator is i32
// (amd_triton_npu/backend/matmul_transform.py:62-64).
//
// Kernel design (one persistent CTA per SM, 6 warps, warp-specialised):
//   warp 0     TMA producer: one elected thread streams 128-byte-wide K slices
//              of A and B into a STAGES-deep shared-memory ring (128B swizzle);
//   warp 1     MMA issuer: allocates TMEM, one thread issues tcgen05.mma for
//              each 32-byte K step and commits each stage back to the producer;
//   warps 2-5  epilogue: tcgen05.ld the accumulator (each warp owns its 32 TMEM
//              lanes = 32 rows), convert, store C with 16-byte stores.
// Tiles are 128 x 256 with two TMEM accumulator buffers (512 columns), so the
// epilogue of one tile overlaps the main loop of the next.  B in row-major
// [K, N] is consumed as an MN-major operand straight from its TMA tile (no
// transpose pass); W in [N, K] is K-major.  Out-of-range rows / columns / K
// are zero-filled by TMA and masked in the epilogue.
//
// int16: A = 256*Ah + Al with Ah = A >> 8 (s8) and Al = A & 255 (u8), likewise
// B.  A@B = 2^16 AhBh + 2^8 (AhBl + AlBh) + AlBl: four kind::i8 MMAs per K step
// into three s32 accumulators (the two cross terms share one), combined in the
// epilogue modulo 2^32 -- exactly the wrap-around of an int32 accumulator.
// The limb planes are produced by a small split kernel into a workspace.
//
// Every mbarrier wait is bounded; a timeout sets a device status word
// (read with xb_device_status) and the kernel drains its in-flight copies and
// MMAs, frees TMEM and returns.
#include "common.cuh"
#include "tc.cuh"

#include <mutex>

namespace xb {
namespace gemm {

using namespace tc;

__device__ int g_gemm_status = 0;
constexpr uint64_t kWaitLimit = 2000000000ull;  // 2 s per wait: far above any legitimate wait

// CTA-pair raster group (in 256-row tiles) and int8 pair ring depth; build-time
// tuning knobs (nvcc -D...), defaults measured best on B200
#ifndef XB_PAIR_GROUP_M
#define XB_PAIR_GROUP_M 8
#endif
#ifndef XB_I8_PAIR_STAGES
#define XB_I8_PAIR_STAGES 6
#endif
// L2 cache policies of the tiled GEMMs: bit 0 = C stores evict-first (C is
// written once), bit 1 = A loads evict-last (an A panel is reused by every
// column tile of its raster group)
#ifndef XB_L2_HINTS
#define XB_L2_HINTS 0
#endif

enum Kind { kBf16 = 0, kInt8 = 1, kInt16Limbs = 2 };
// kOutSwiglu: W interleaves 64-row blocks of gate and up rows (block 2b =
// gate rows 64b.., block 2b+1 = up rows 64b..), so a 256-column tile holds
// the gate and up values of 128 output features (and a 128-row block of W,
// the decode kernel's unit, those of 64); the epilogue writes
// bf16(silu(bf16(g)) * bf16(u)) into C [M, N/2] -- the roundings of two bf16
// linears followed by the silu*up kernel.
// kOutArgmax (swap-AB only): no logits; per 128-row tile of W and token the
// best (value, row) goes to C as {float, int32} [row tiles][tokens], and
// xb_linear_argmax_bf16 reduces the tiles (the greedy next token).
// kOutQkv: the fused QKV projection of a prefill, finished in the epilogue:
// bf16(acc + bias) per 64-column head slot, RoPE of the query / key heads
// (none without tables), written to q [B, H, S, 64] and the K / V caches at
// pos_offset + s -- the roundings of a linear followed by the RoPE kernel.
enum Out { kOutF32 = 0, kOutBf16 = 1, kOutI32 = 2, kOutSwiglu = 3, kOutArgmax = 4, kOutQkv = 5 };

constexpr int tmem_cols_for(int cols) { return cols <= 32 ? 32 : cols <= 64 ? 64 : cols <= 128 ? 128 : cols <= 256 ? 256 : 512; }

// BN_: tile N (0 = the default for the kind).  The small-M path (swap-AB:
// weight rows in the 128-row MMA dimension, up to 64 tokens in N) uses 64
// with a deeper ring, since it streams weights from HBM in short K ranges.
// PAIR: a cluster of two CTAs computes one 256 x BN tile with cta_group::2
// MMAs; each CTA stages its own 128 rows of A and half of the B columns, so
// a CTA moves 2/3 of the operand bytes of a 128 x 256 single-CTA tile for
// the same MMA work (the L2 -> shared-memory stream is what bounds the
// single-CTA kernel at large shapes).
template <int KIND, bool B_KMAJOR, int BN_ = 0, bool PAIR = false>
struct Cfg {
  static constexpr int BM = 128;                    // rows per CTA (TMEM lanes)
  static constexpr int TILE_M = PAIR ? 256 : 128;   // rows per tile
  static constexpr int BN = BN_ ? BN_ : (KIND == kInt16Limbs ? 128 : 256);
  static constexpr int BN_CTA = PAIR ? BN / 2 : BN;  // B columns staged per CTA
  static constexpr int ESZ = KIND == kBf16 ? 2 : 1;  // operand element bytes
  static constexpr int BK = 128 / ESZ;              // K elements per stage (128 bytes)
  static constexpr int PLANES = KIND == kInt16Limbs ? 2 : 1;
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BN_CTA * 128;
  static constexpr int STAGE_BYTES = PLANES * (A_BYTES + B_BYTES);
  // BN <= 64 (small-M, swap-AB): 6 slots leave room on the SM for the small
  // kernel before it, so the weight prefetch can overlap that kernel
  static constexpr int STAGES = PAIR ? (KIND == kInt16Limbs ? 4 : KIND == kInt8 ? XB_I8_PAIR_STAGES : 6)
                                     : KIND == kInt16Limbs ? 3 : (BN <= 64 ? 6 : 4);
  static constexpr int UMMA_K = 32 / ESZ;  // 32 bytes of K per MMA
  static constexpr int KSTEPS = BK / UMMA_K;
  static constexpr int ACCS = KIND == kInt16Limbs ? 3 : 1;
  static constexpr int ACC_BUFS = KIND == kInt16Limbs ? 1 : 2;
  static constexpr int TMEM_COLS = tmem_cols_for(ACCS * ACC_BUFS * BN);
  static constexpr int B_BOX_N = 128 / ESZ;  // N elements in one MN-major B box
  static constexpr int B_BOXES = B_KMAJOR ? 1 : BN_CTA / B_BOX_N;
  static constexpr int B_BOX_BYTES = B_KMAJOR ? B_BYTES : BK * 128;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024;
  static_assert(ACCS * ACC_BUFS * BN <= TMEM_COLS, "TMEM budget");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(B_KMAJOR || BN_CTA % B_BOX_N == 0, "MN-major B needs whole boxes");
};

struct alignas(64) Maps {
  CUtensorMap a[2];  // A plane(s): [M, K] K-major
  CUtensorMap b[2];  // B plane(s): [K, N] MN-major, or W [N, K] K-major
  CUtensorMap c;     // C [M, N] for the TMA-store epilogue (4-byte outputs), 32 x 32 boxes
};

// Epilogue staging for TMA stores: per epilogue warp two 32 x 32 4-byte
// tiles (128-byte rows, 128-byte swizzle), after the operand ring.
constexpr int kEpiStageBytes = 4 * 2 * 32 * 128;

struct Args {
  void* c;
  const void* bias;  // bf16 [N] or nullptr (linear layer only)
  const void* residual;  // bf16 [M, N] added after the bf16 rounding (bf16 output), or nullptr
  int64_t ldr;
  int act;  // bf16 output: 1 = tanh GELU of the bf16-rounded linear output (GPT-2 c_fc)
  int64_t ldc;
  int64_t split_stride;  // elements between the split-K slices of c
  int m, n, k;
  int tiles_m, tiles_n, num_tiles, kblocks;
  int splits, kps;  // split-K: `splits` slices of `kps` K blocks each
  // N-sharded GEMM over the GPUs of a node: the epilogue stores every tile
  // into each rank's C (peer pointers, this rank's column block), and the
  // grid's last CTA signals every peer.
  int c_tma;  // 1: C is written through maps.c (TMA stores from shared memory)
  // kOutQkv: destinations, head layout and RoPE tables (rows are the B*S tokens)
  void* q_out;
  void* k_cache;
  void* v_cache;
  const float* cos_t;
  const float* sin_t;
  int H, KVH, S, smax, pos;
  int rope_dup;  // 1: every table row's second half repeats its first (read the first only)
  int world, rank;
  void* peers[8];
  uint64_t* signals[8];  // each rank's signal buffer (uint64 [2 * world + 1], layout in peer.cu)
  uint64_t epoch;        // 1-based number of this sharded call on this rank
  uint64_t peer_timeout_ns;  // limit of the wait for a peer's release of its C
};

constexpr int kGroupM = 16;  // tile raster: groups of 16 M-tiles sweep N (L2 reuse)

template <int GROUP_M = kGroupM>
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& tm, int& tn) {
  const int group = GROUP_M * tiles_n;
  const int g = t / group;
  const int first_m = g * GROUP_M;
  const int gm = min(GROUP_M, tiles_m - first_m);
  const int r = t - g * group;
  tm = first_m + r % gm;
  tn = r / gm;
}

// TRANS: the epilogue stores C^T (element (r, c) of the tile product at
// c * ldc + r); with A = W and B = X this computes Y = X W^T for few tokens.
__device__ __forceinline__ void red_release_sys_add(uint64_t* p, uint64_t v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Sharded GEMM: before this rank's first store into peer pe's C, peer pe
// must have released the previous call's C, i.e. its own stream must have
// reached this call's GEMM (which releases at its start, after every earlier
// kernel on that stream -- the readers of the previous C -- completed).
// Polls this rank's own signal buffer (peers write their release counts into
// it); false when a peer has not released within the call's time limit.
__device__ __forceinline__ bool wait_peer_releases(const Args& args) {
  const uint64_t* rel = args.signals[args.rank] + args.world + 1;
  const uint64_t t0 = globaltimer_ns();
  for (int pe = 0; pe < args.world; ++pe) {
    if (pe == args.rank) continue;
    while (ld_acquire_sys_u64(rel + pe) < args.epoch) {
      if (globaltimer_ns() - t0 > args.peer_timeout_ns) return false;
      __nanosleep(256);
    }
  }
  return true;
}

// EPI: epilogue warps (4, or 8 for bf16-output and fused-QKV tiles: two warps
// per TMEM lane quarter, each finishing half of the tile's 32-column chunks,
// so that a short-K tile's epilogue hides behind the next tile's main loop).
template <int KIND, bool B_KMAJOR, int OUT, int BN_ = 0, bool TRANS = false, bool PEERS = false, bool PAIR = false,
          int EPI = 4>
__global__ void __launch_bounds__(64 + 32 * EPI, 1) gemm_kernel(const __grid_constant__ Maps maps, const Args args) {
  using C = Cfg<KIND, B_KMAJOR, BN_, PAIR>;
  static_assert(EPI == 4 || (EPI == 8 && (OUT == kOutBf16 || OUT == kOutQkv) && !TRANS && !PEERS),
                "eight epilogue warps: bf16-output or fused-QKV row-major tiles only");
  constexpr int kEpiThreads = 32 * EPI;
  constexpr int kHalves = EPI / 4;  // warps per TMEM lane quarter
  constexpr int GM = PAIR ? XB_PAIR_GROUP_M : kGroupM;  // raster group (in tiles)
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[C::STAGES];
  __shared__ __align__(8) uint64_t empty_bar[C::STAGES];
  __shared__ __align__(8) uint64_t tfull_bar[C::ACC_BUFS];
  __shared__ __align__(8) uint64_t tempty_bar[C::ACC_BUFS];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t base_u32 = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - smem_u32(smem_raw));
  // Pair roles: CTA 0 of the cluster issues the MMAs and owns the barriers
  // that gate them; both CTAs load operands and run an epilogue.
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = crank == 0;
  const int tile0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tstep = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < C::ACC_BUFS; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], PAIR ? 2 * kEpiThreads : kEpiThreads);
    }
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    for (int p = 0; p < C::PLANES; ++p) {
      prefetch_tmap(&maps.a[p]);
      prefetch_tmap(&maps.b[p]);
    }
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc2(&tmem_base_sh, C::TMEM_COLS);
      tmem_relinquish2();
    } else {
      tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR) cluster_sync();  // barrier init and TMEM allocation visible to the peer CTA
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  // Everything above touched only shared memory, TMEM and the tensor maps in
  // the kernel parameters: it overlaps the previous kernel on the stream.
  // The small-M producer first issues the weight loads of its first ring
  // slots (weights are never written by an earlier kernel), then waits.
  constexpr bool kPrefetchW = TRANS && !PAIR;
  if (!(kPrefetchW && threadIdx.x == 0)) {
    pdl_wait();
    pdl_trigger();
  }

  auto fail = [&]() {
    atomicExch(&g_gemm_status, XB_ERR_TIMEOUT);
    abort_flag = 1;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t it = 0;  // global k-block counter (ring position)
      uint32_t issued[C::STAGES];  // loads issued per stage (for the exit drain)
#pragma unroll
      for (int s = 0; s < C::STAGES; ++s) issued[s] = 0;
      bool ok = true;
      int npre = 0;  // ring slots whose weight (A) tile was issued before the wait
      if constexpr (kPrefetchW) {
        if (tile0 < args.num_tiles) {
          int tm, tn;
          tile_coords<GM>(tile0 / args.splits, args.tiles_m, args.tiles_n, tm, tn);
          const int kb0 = (tile0 % args.splits) * args.kps;
          npre = min(C::STAGES, min(kb0 + args.kps, args.kblocks) - kb0);
          for (int i = 0; i < npre; ++i) {
            mbar_arrive_expect_tx(&full_bar[i], C::STAGE_BYTES);
            tma_load_2d(smem + i * C::STAGE_BYTES, &maps.a[0], &full_bar[i], (kb0 + i) * C::BK, tm * C::BM);
          }
        }
        pdl_wait();
        pdl_trigger();
      }
      for (int t = tile0; t < args.num_tiles && ok; t += tstep) {
        int tm, tn;
        tile_coords<GM>(t / args.splits, args.tiles_m, args.tiles_n, tm, tn);
        const int kb0 = (t % args.splits) * args.kps;
        const int kb1 = min(kb0 + args.kps, args.kblocks);
        const int arow = tm * C::TILE_M + (int)crank * C::BM;    // this CTA's rows of A
        const int bcol = tn * C::BN + (int)crank * C::BN_CTA;    // this CTA's columns of B
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          const bool pre = (int)it < npre;  // slot armed and its A tile issued before the wait
          const bool got = pre || (PAIR ? mbar_wait_cl(&empty_bar[s], ph ^ 1, kWaitLimit, &abort_flag)
                                        : mbar_wait(&empty_bar[s], ph ^ 1, kWaitLimit, &abort_flag));
          if (!got) { fail(); ok = false; break; }
          // the leader's full barrier counts the bytes of both CTAs of a pair
          if (leader && !pre) mbar_arrive_expect_tx(&full_bar[s], (PAIR ? 2 : 1) * C::STAGE_BYTES);
          const uint32_t fb = PAIR ? mapa_u32(smem_u32(&full_bar[s]), 0) : 0u;
          auto load = [&](void* dst, const CUtensorMap* map, int32_t c0, int32_t c1) {
            if constexpr (PAIR) tma_load_2d_pair(dst, map, fb, c0, c1);
            else tma_load_2d(dst, map, &full_bar[s], c0, c1);
          };
          auto load_a = [&](void* dst, const CUtensorMap* map, int32_t c0, int32_t c1) {
            if constexpr ((XB_L2_HINTS & 2) != 0 && !TRANS) {
              if constexpr (PAIR) tma_load_2d_pair_hint(dst, map, fb, c0, c1, l2_policy_evict_last());
              else tma_load_2d_hint(dst, map, &full_bar[s], c0, c1, l2_policy_evict_last());
            } else {
              load(dst, map, c0, c1);
            }
          };
          uint8_t* st = smem + s * C::STAGE_BYTES;
          for (int p = 0; p < C::PLANES; ++p) {
            if (!pre) load_a(st + p * C::A_BYTES, &maps.a[p], kb * C::BK, arow);
            uint8_t* sb = st + C::PLANES * C::A_BYTES + p * C::B_BYTES;
            if (B_KMAJOR) {
              load(sb, &maps.b[p], kb * C::BK, bcol);
            } else {
#pragma unroll
              for (int j = 0; j < C::B_BOXES; ++j) load(sb + j * C::B_BOX_BYTES, &maps.b[p], bcol + j * C::B_BOX_N, kb * C::BK);
            }
          }
          issued[s] = it / C::STAGES + 1;
        }
      }
      if (leader) {
        // Drain: every load issued into a stage must have landed before exit
        // (also after an abort; one time limit for all stages).
        uint64_t deadline = 0;
        for (int s = 0; s < C::STAGES; ++s)
          if (issued[s] && !mbar_wait_deadline(&full_bar[s], (issued[s] - 1) & 1, &deadline, kWaitLimit)) fail();
      } else if (!ok) {
        // The odd CTA's loads complete on the leader's barriers: after a
        // failure give any load still in flight time to land (loads take
        // microseconds) before the cluster barrier lets the CTA exit.
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 1000000ull) __nanosleep(1000);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      bool any = false;
      // commit to a barrier of this CTA and, for a pair, to the same barrier of the odd CTA
      auto commit = [&](uint64_t* bar) {
        if constexpr (PAIR) {
          tc_commit2(smem_u32(bar));
          tc_commit2(mapa_u32(smem_u32(bar), 1));
        } else {
          tc_commit(bar);
        }
      };
      for (int t = tile0; t < args.num_tiles && ok; t += tstep, ++local) {
        const int buf = local % C::ACC_BUFS;
        const uint32_t tph = (local / C::ACC_BUFS) & 1;
        const bool got = PAIR ? mbar_wait_cl(&tempty_bar[buf], tph ^ 1, kWaitLimit, &abort_flag)
                              : mbar_wait(&tempty_bar[buf], tph ^ 1, kWaitLimit, &abort_flag);
        if (!got) { fail(); break; }
        tc_fence_after();
        const uint32_t d0 = tmem_base + buf * C::ACCS * C::BN;
        const int kb0 = (t % args.splits) * args.kps;
        const int kb1 = min(kb0 + args.kps, args.kblocks);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&full_bar[s], ph, kWaitLimit, &abort_flag)) { fail(); ok = false; break; }
          tc_fence_after();
          const uint32_t st = base_u32 + s * C::STAGE_BYTES;
#pragma unroll
          for (int ks = 0; ks < C::KSTEPS; ++ks) {
            const uint32_t acc = (kb > kb0 || ks > 0) ? 1u : 0u;
            uint64_t ad[2], bd[2];
#pragma unroll
            for (int p = 0; p < C::PLANES; ++p) {
              ad[p] = umma_desc_sw128(st + p * C::A_BYTES + ks * 32, 16, 1024);
              const uint32_t sb = st + C::PLANES * C::A_BYTES + p * C::B_BYTES;
              bd[p] = B_KMAJOR ? umma_desc_sw128(sb + ks * 32, 16, 1024)
                               : umma_desc_sw128(sb + ks * C::UMMA_K * 128, C::B_BOX_BYTES, 1024);
            }
            constexpr uint32_t bmn = B_KMAJOR ? 0 : 1;
            if constexpr (PAIR && KIND == kBf16) {
              mma2_f16(d0, ad[0], bd[0], umma_idesc(1, 1, 1, 0, bmn, C::TILE_M, C::BN), acc);
            } else if constexpr (PAIR && KIND == kInt8) {
              mma2_i8(d0, ad[0], bd[0], umma_idesc(2, 1, 1, 0, bmn, C::TILE_M, C::BN), acc);
            } else if constexpr (PAIR) {  // int16 limbs, as below, on the 256-row pair tile
              mma2_i8(d0, ad[0], bd[0], umma_idesc(2, 1, 1, 0, bmn, C::TILE_M, C::BN), acc);
              mma2_i8(d0 + C::BN, ad[0], bd[1], umma_idesc(2, 1, 0, 0, bmn, C::TILE_M, C::BN), acc);
              mma2_i8(d0 + C::BN, ad[1], bd[0], umma_idesc(2, 0, 1, 0, bmn, C::TILE_M, C::BN), 1u);
              mma2_i8(d0 + 2 * C::BN, ad[1], bd[1], umma_idesc(2, 0, 0, 0, bmn, C::TILE_M, C::BN), acc);
            } else if constexpr (KIND == kBf16) {
              mma_f16(d0, ad[0], bd[0], umma_idesc(1, 1, 1, 0, bmn, C::BM, C::BN), acc);
            } else if constexpr (KIND == kInt8) {
              mma_i8(d0, ad[0], bd[0], umma_idesc(2, 1, 1, 0, bmn, C::BM, C::BN), acc);
            } else {
              // planes: 0 = high limb (s8), 1 = low limb (u8)
              mma_i8(d0, ad[0], bd[0], umma_idesc(2, 1, 1, 0, bmn, C::BM, C::BN), acc);               // hi*hi
              mma_i8(d0 + C::BN, ad[0], bd[1], umma_idesc(2, 1, 0, 0, bmn, C::BM, C::BN), acc);       // hi*lo
              mma_i8(d0 + C::BN, ad[1], bd[0], umma_idesc(2, 0, 1, 0, bmn, C::BM, C::BN), 1u);        // lo*hi
              mma_i8(d0 + 2 * C::BN, ad[1], bd[1], umma_idesc(2, 0, 0, 0, bmn, C::BM, C::BN), acc);   // lo*lo
            }
            any = true;
          }
          commit(&empty_bar[s]);  // frees the stage once these MMAs have read it
        }
        if (!ok) break;
        commit(&tfull_bar[buf]);  // accumulator ready for the epilogue
      }
      if (any) {
        if constexpr (PAIR) tc_commit2(smem_u32(&drain_bar));
        else tc_commit(&drain_bar);
        // every issued MMA has completed before TMEM is released (also after an abort)
        uint64_t deadline = 0;
        if (!mbar_wait_deadline(&drain_bar, 0, &deadline, kWaitLimit)) fail();
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int ew = warp - 2;  // epilogue warp 0 .. EPI - 1
    const int half = ew >> 2;  // which of the quarter's warps (EPI = 8)
    int local = 0;
    int first_tile = tile0;
    if constexpr (PEERS) {
      // CTA 0 tells every peer that this rank's C is free for this call
      // (everything before this kernel on the stream has completed).
      if (blockIdx.x == 0 && warp == 2 && lane == 0)
        for (int pe = 0; pe < args.world; ++pe)
          if (pe != args.rank) red_release_sys_add(args.signals[pe] + args.world + 1 + args.rank, 1ull);
      bool ok = true;
      if (lane == 0) ok = wait_peer_releases(args);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) {
        fail();
        first_tile = args.num_tiles;  // no tile of this warp is stored anywhere
      }
    }
    for (int t = first_tile; t < args.num_tiles; t += tstep, ++local) {
      const int buf = local % C::ACC_BUFS;
      const uint32_t tph = (local / C::ACC_BUFS) & 1;
      const bool got = PAIR ? mbar_wait_cl(&tfull_bar[buf], tph, kWaitLimit, &abort_flag)
                            : mbar_wait(&tfull_bar[buf], tph, kWaitLimit, &abort_flag);
      if (!got) {
        fail();
        // the argmax epilogue's warps meet at named barriers every tile: after a
        // timeout they keep stepping through the tiles (garbage, flagged) so
        // none waits for a warp that left
        if constexpr (OUT != kOutArgmax) break;
      }
      tc_fence_after();
      int tm, tn;
      tile_coords<GM>(t / args.splits, args.tiles_m, args.tiles_n, tm, tn);
      const int row = tm * C::TILE_M + (int)crank * C::BM + q * 32 + lane;
      const int64_t slice = (int64_t)(t % args.splits) * args.split_stride;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + buf * C::ACCS * C::BN;
#pragma unroll 1
      for (int cc = 0; cc < C::BN / 32; ++cc) {
        if constexpr (kHalves > 1) {  // chunks (QKV: 64-column head slots) alternate between the quarter's warps
          if ((((OUT == kOutQkv) ? (cc >> 1) : cc) % kHalves) != half) continue;
        }
        if constexpr (OUT == kOutQkv) {
          static_assert(!TRANS && !PEERS && C::BN % 64 == 0, "fused QKV epilogue: row-major tiles of whole heads");
          if (cc & 1) continue;  // the even chunk takes the whole 64-column head slot
          uint32_t v0[32], v1[32];
          tmem_ld_32x32b_x32(tbase + cc * 32, v0);
          tmem_ld_32x32b_x32(tbase + cc * 32 + 32, v1);
          tmem_ld_wait();
          const int c0 = tn * C::BN + cc * 32;  // first column of the head slot
          const int row0 = row - lane;
          if (row0 >= args.m || c0 >= args.n) continue;  // warp-uniform
          const int slot = c0 >> 6;
          const __nv_bfloat16* bp = static_cast<const __nv_bfloat16*>(args.bias);
          float x0[32], x1[32];
          if (bp && (reinterpret_cast<uintptr_t>(bp + c0) & 15) == 0) {
            // the head slot's 64 bias values as eight 16-byte loads (the same
            // address in every lane)
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              const uint4 r0 = __ldg(reinterpret_cast<const uint4*>(bp + c0 + j));
              const uint4 r1 = __ldg(reinterpret_cast<const uint4*>(bp + c0 + 32 + j));
              const __nv_bfloat16* b0 = reinterpret_cast<const __nv_bfloat16*>(&r0);
              const __nv_bfloat16* b1 = reinterpret_cast<const __nv_bfloat16*>(&r1);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                x0[j + e] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(v0[j + e]) + __bfloat162float(b0[e])));
                x1[j + e] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(v1[j + e]) + __bfloat162float(b1[e])));
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float b0 = bp ? __bfloat162float(bp[c0 + j]) : 0.0f;
              const float b1 = bp ? __bfloat162float(bp[c0 + 32 + j]) : 0.0f;
              x0[j] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(v0[j]) + b0));
              x1[j] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(v1[j]) + b1));
            }
          }
          // destination row of token `rw` (its head slot: the query output or
          // the K / V cache at the token's position)
          auto dst_of = [&](int rw) -> __nv_bfloat16* {
            const int bq = rw / args.S, sq = rw - bq * args.S;
            if (slot < args.H)
              return static_cast<__nv_bfloat16*>(args.q_out) + (((int64_t)bq * args.H + slot) * args.S + sq) * 64;
            if (slot < args.H + args.KVH)
              return static_cast<__nv_bfloat16*>(args.k_cache) +
                     (((int64_t)bq * args.KVH + (slot - args.H)) * args.smax + args.pos + sq) * 64;
            return static_cast<__nv_bfloat16*>(args.v_cache) +
                   (((int64_t)bq * args.KVH + (slot - args.H - args.KVH)) * args.smax + args.pos + sq) * 64;
          };
          // the warp's 32 rows x 128 bytes (bf16(x W^T + b), exact in bf16)
          // through its swizzled staging tile; RoPE is applied on the way out,
          // where four lanes share a token: lane (r, pc) rotates the pairs
          // (8 pc + e, 32 + 8 pc + e) of row r and stores both 16-byte pieces,
          // so the table rows are read in 32-byte runs and every store
          // instruction writes eight tokens' half rows
          uint8_t* stg = smem + C::STAGES * C::STAGE_BYTES + (EPI == 4 ? q * 2 : ew) * (32 * 128);
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            __nv_bfloat162 h0[4], h1[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              h0[e] = __floats2bfloat162_rn(x0[j + 2 * e], x0[j + 2 * e + 1]);
              h1[e] = __floats2bfloat162_rn(x1[j + 2 * e], x1[j + 2 * e + 1]);
            }
            const int p0 = j / 8, p1 = 4 + j / 8;  // 16-byte pieces of the row
            *reinterpret_cast<int4*>(stg + lane * 128 + ((p0 ^ (lane & 7)) * 16)) = *reinterpret_cast<int4*>(h0);
            *reinterpret_cast<int4*>(stg + lane * 128 + ((p1 ^ (lane & 7)) * 16)) = *reinterpret_cast<int4*>(h1);
          }
          __syncwarp();
          const bool rope = args.cos_t && slot < args.H + args.KVH;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int r = k * 8 + lane / 4, pc = lane % 4;
            const int rw = row0 + r;
            int4 a0 = *reinterpret_cast<const int4*>(stg + r * 128 + ((pc ^ (r & 7)) * 16));
            int4 a1 = *reinterpret_cast<const int4*>(stg + r * 128 + (((pc + 4) ^ (r & 7)) * 16));
            if (rw >= args.m) continue;
            if (rope) {
              const int pos = args.pos + (rw - (rw / args.S) * args.S);
              const float4* cr = reinterpret_cast<const float4*>(args.cos_t + (int64_t)pos * 64 + pc * 8);
              const float4* sr = reinterpret_cast<const float4*>(args.sin_t + (int64_t)pos * 64 + pc * 8);
              const float4 ca0 = __ldg(cr), ca1 = __ldg(cr + 1), sa0 = __ldg(sr), sa1 = __ldg(sr + 1);
              const float4 cb0 = args.rope_dup ? ca0 : __ldg(cr + 8), cb1 = args.rope_dup ? ca1 : __ldg(cr + 9);
              const float4 sb0 = args.rope_dup ? sa0 : __ldg(sr + 8), sb1 = args.rope_dup ? sa1 : __ldg(sr + 9);
              const float c0v[8] = {ca0.x, ca0.y, ca0.z, ca0.w, ca1.x, ca1.y, ca1.z, ca1.w};
              const float c1v[8] = {cb0.x, cb0.y, cb0.z, cb0.w, cb1.x, cb1.y, cb1.z, cb1.w};
              const float s0v[8] = {sa0.x, sa0.y, sa0.z, sa0.w, sa1.x, sa1.y, sa1.z, sa1.w};
              const float s1v[8] = {sb0.x, sb0.y, sb0.z, sb0.w, sb1.x, sb1.y, sb1.z, sb1.w};
              __nv_bfloat16* h0 = reinterpret_cast<__nv_bfloat16*>(&a0);
              __nv_bfloat16* h1 = reinterpret_cast<__nv_bfloat16*>(&a1);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float u0 = __bfloat162float(h0[e]), u1 = __bfloat162float(h1[e]);
                const float y0 = __fadd_rn(__fmul_rn(u0, c0v[e]), __fmul_rn(-u1, s0v[e]));
                const float y1 = __fadd_rn(__fmul_rn(u1, c1v[e]), __fmul_rn(u0, s1v[e]));
                h0[e] = __float2bfloat16_rn(y0);
                h1[e] = __float2bfloat16_rn(y1);
              }
            }
            __nv_bfloat16* d = dst_of(rw);
            *reinterpret_cast<int4*>(d + pc * 8) = a0;
            *reinterpret_cast<int4*>(d + 32 + pc * 8) = a1;
          }
          __syncwarp();  // staging free for the next head slot
          continue;
        }
        if constexpr (OUT == kOutSwiglu) {
          if (cc >= C::BN / 64) continue;
          uint32_t gv[32], uv[32];
          const int gc = (cc >> 1) * 128 + (cc & 1) * 32;  // 64 gate columns, then their 64 up columns
          tmem_ld_32x32b_x32(tbase + gc, gv);        // gate features
          tmem_ld_32x32b_x32(tbase + gc + 64, uv);   // up features
          tmem_ld_wait();
          const int f0 = tn * (C::BN / 2) + cc * 32;  // output feature of column 0
          const int nout = args.n / 2;
          if (row >= args.m || f0 >= nout) continue;
          __nv_bfloat16* cp = static_cast<__nv_bfloat16*>(args.c) + (int64_t)row * args.ldc + f0;
          float o[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float g = __bfloat162float(__float2bfloat16_rn(__uint_as_float(gv[j])));
            const float u = __bfloat162float(__float2bfloat16_rn(__uint_as_float(uv[j])));
            o[j] = __fmul_rn(silu_bf16path(g), u);
          }
          if (f0 + 32 <= nout && ((reinterpret_cast<uintptr_t>(cp) & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              __nv_bfloat162 h[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(o[j + 2 * e], o[j + 2 * e + 1]);
              *reinterpret_cast<int4*>(cp + j) = *reinterpret_cast<int4*>(h);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (f0 + j < nout) cp[j] = __float2bfloat16_rn(o[j]);
          }
          continue;
        }
        uint32_t v[32];
        tmem_ld_32x32b_x32(tbase + cc * 32, v);
        if constexpr (KIND == kInt16Limbs) {
          uint32_t mid[32], lo[32];
          tmem_ld_32x32b_x32(tbase + C::BN + cc * 32, mid);
          tmem_ld_32x32b_x32(tbase + 2 * C::BN + cc * 32, lo);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = (v[j] << 16) + (mid[j] << 8) + lo[j];
        } else {
          tmem_ld_wait();
        }
        const int col0 = tn * C::BN + cc * 32;
        if constexpr (OUT == kOutArgmax) {
          static_assert(TRANS && !PAIR && !PEERS && C::BN == 64, "argmax epilogue: swap-AB, 64 tokens per tile");
          // Warp q transposes its 32 rows x 32 tokens through shared memory so
          // lane j scans token col0 + j down the rows in order; the four
          // warps' candidates meet in shared memory after the last chunk.
          float* stg = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES);
          float* cv = stg + 4 * 32 * 33;                // [warp quarter][64 tokens]
          int* ci = reinterpret_cast<int*>(cv + 4 * 64);
#pragma unroll
          for (int j = 0; j < 32; ++j) stg[(q * 32 + lane) * 33 + j] = __uint_as_float(v[j]);
          __syncwarp();
          // rows in increasing order: a later row replaces the best only if
          // strictly larger, or the first NaN (argmax_better's order)
          float best = 0.0f;
          int bi = args.m;  // no candidate
          const int rmax = min(32, args.m - (row - lane));
#pragma unroll 8
          for (int r = 0; r < rmax; ++r) {
            const float val = stg[(q * 32 + r) * 33 + lane];
            if (bi == args.m || val > best || (val != val && best == best)) {
              best = val;
              bi = row - lane + r;
            }
          }
          cv[q * 64 + cc * 32 + lane] = best;
          ci[q * 64 + cc * 32 + lane] = bi;
          __syncwarp();
          if (cc == C::BN / 32 - 1) {
            asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
            if (q == 0) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int tk = h * 32 + lane;
                float b = cv[tk];
                int i = ci[tk];
#pragma unroll
                for (int w = 1; w < 4; ++w)
                  if (argmax_better(b, i, cv[w * 64 + tk], ci[w * 64 + tk], args.m)) {
                    b = cv[w * 64 + tk];
                    i = ci[w * 64 + tk];
                  }
                const int token = tn * C::BN + tk;
                if (token < args.n)
                  static_cast<uint2*>(args.c)[(int64_t)tm * args.n + token] = make_uint2(__float_as_uint(b), (uint32_t)i);
              }
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");  // candidates read: free for the next tile
          }
          continue;
        }
        if constexpr (OUT != kOutBf16 && !TRANS && !PEERS) {
          if (args.c_tma) {
            // Coalesced store: each thread writes its row's 128 bytes into a
            // swizzled 32 x 32 staging tile, one lane stores the tile with TMA
            // (the unit clips rows / columns outside C).  Chunks wholly outside
            // C (warp-uniform test) touch no staging buffer and commit nothing.
            if (col0 >= args.n || row - lane >= args.m) continue;
            if constexpr (OUT == kOutF32) {
              if (args.bias) {
                const __nv_bfloat16* bp = static_cast<const __nv_bfloat16*>(args.bias);
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (col0 + j < args.n) v[j] = __float_as_uint(__uint_as_float(v[j]) + __bfloat162float(bp[col0 + j]));
              }
            }
            uint8_t* stg = smem + C::STAGES * C::STAGE_BYTES + (q * 2 + (cc & 1)) * (32 * 128);
            // the store that last used this buffer has read it (a tile's first
            // chunk waits for all: chunks past the edges of C commit nothing)
            if (lane == 0) {
              if (cc == 0) bulk_wait_read<0>();
              else bulk_wait_read<1>();
            }
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 8; ++j)
              *reinterpret_cast<uint4*>(stg + lane * 128 + ((j ^ (lane & 7)) * 16)) =
                  make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if constexpr ((XB_L2_HINTS & 1) != 0) tma_store_2d_hint(&maps.c, stg, col0, row, l2_policy_evict_first());
              else tma_store_2d(&maps.c, stg, col0, row);
              bulk_commit();
            }
            continue;
          }
        }
        if constexpr (TRANS && !PEERS) {
          if (args.c_tma) {
            // C^T through shared memory: thread `lane` (one output feature)
            // writes its 32 token values down a column of a [32 tokens][32
            // features] staging tile -- consecutive lanes, consecutive
            // addresses -- and one lane stores the tile with TMA (3-D map:
            // features, tokens, K slice; the unit clips the edges).
            const int frow0 = row - lane;
            if (col0 >= args.n || frow0 >= args.m) continue;  // warp-uniform
            if (args.bias && row < args.m) {
              const float bv = __bfloat162float(static_cast<const __nv_bfloat16*>(args.bias)[row]);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + bv);
            }
            if (OUT == kOutBf16 && args.act == 1) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                v[j] = __float_as_uint(gelu_tanh_bf16path(__bfloat162float(__float2bfloat16_rn(__uint_as_float(v[j])))));
            }
            uint8_t* stg = smem + C::STAGES * C::STAGE_BYTES + (q * 2 + (cc & 1)) * (32 * 128);
            if (lane == 0) {
              if (cc == 0) bulk_wait_read<0>();
              else bulk_wait_read<1>();
            }
            __syncwarp();
            if constexpr (OUT == kOutBf16) {
              __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(stg);
#pragma unroll
              for (int j = 0; j < 32; ++j) st[j * 32 + lane] = __float2bfloat16_rn(__uint_as_float(v[j]));
            } else {
              uint32_t* st = reinterpret_cast<uint32_t*>(stg);
#pragma unroll
              for (int j = 0; j < 32; ++j) st[j * 32 + lane] = v[j];
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&maps.c, stg, frow0, col0, t % args.splits);
              bulk_commit();
            }
            continue;
          }
        }
        if constexpr ((PEERS || OUT == kOutBf16) && !TRANS) {
          if (args.c_tma) {
            // Stores of whole lines: the warp's 32 x 32 chunk goes through a
            // swizzled staging tile, then each store instruction writes
            // complete 128-byte (int32) or 64-byte (bf16) row segments of 4 or
            // 8 rows -- to C, or with peers to this rank's C and over NVLink to
            // every peer's.
            const int row0 = row - lane;
            if (col0 >= args.n || row0 >= args.m) continue;  // warp-uniform
            if (col0 + 32 <= args.n) {
              // residual pieces this lane adds on the way out (row k * 8 + lane / 4,
              // 16-byte piece lane % 4): requested now, eight rows' 64-byte
              // segments per load instruction, used after the staging
              int4 rres[4];
              if constexpr (OUT == kOutBf16 && !PEERS) {
                if (args.residual) {
#pragma unroll
                  for (int k = 0; k < 4; ++k) {
                    const int r = k * 8 + lane / 4;
                    rres[k] = row0 + r < args.m
                                  ? __ldg(reinterpret_cast<const int4*>(static_cast<const __nv_bfloat16*>(args.residual) +
                                                                        (int64_t)(row0 + r) * args.ldr + col0 +
                                                                        (lane % 4) * 8))
                                  : make_int4(0, 0, 0, 0);
                  }
                }
              }
              if constexpr (OUT == kOutBf16 && !PEERS) {
                if (args.bias) {
                  const __nv_bfloat16* bp = static_cast<const __nv_bfloat16*>(args.bias);
#pragma unroll
                  for (int j = 0; j < 32; ++j)
                    v[j] = __float_as_uint(__uint_as_float(v[j]) + __bfloat162float(bp[col0 + j]));
                }
                if (args.act == 1) {
#pragma unroll
                  for (int j = 0; j < 32; ++j)
                    v[j] = __float_as_uint(gelu_tanh_bf16path(
                        __bfloat162float(__float2bfloat16_rn(__uint_as_float(v[j])))));
                }
                // (a residual is added on the way out, below: residual + bf16(x W^T + b))
              }
              uint8_t* stg = smem + C::STAGES * C::STAGE_BYTES + (EPI == 4 ? q * 2 : ew) * (32 * 128);
              if constexpr (OUT == kOutBf16) {
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                  __nv_bfloat162 h[4];
#pragma unroll
                  for (int e = 0; e < 4; ++e)
                    h[e] = __floats2bfloat162_rn(__uint_as_float(v[8 * p + 2 * e]),
                                                 __uint_as_float(v[8 * p + 2 * e + 1]));
                  *reinterpret_cast<int4*>(stg + lane * 64 + ((p ^ ((lane >> 1) & 3)) * 16)) =
                      *reinterpret_cast<int4*>(h);
                }
              } else {
#pragma unroll
                for (int p = 0; p < 8; ++p)
                  *reinterpret_cast<uint4*>(stg + lane * 128 + ((p ^ (lane & 7)) * 16)) =
                      make_uint4(v[4 * p], v[4 * p + 1], v[4 * p + 2], v[4 * p + 3]);
              }
              __syncwarp();
              constexpr int kRowsPer = OUT == kOutBf16 ? 8 : 4;      // rows per store instruction
              constexpr int kPieces = OUT == kOutBf16 ? 4 : 8;       // 16-byte pieces per row
              constexpr int kEsz = OUT == kOutBf16 ? 2 : 4;
#pragma unroll 1
              for (int pe = 0; pe < (PEERS ? args.world : 1); ++pe) {
                uint8_t* cb = static_cast<uint8_t*>(PEERS ? args.peers[pe] : args.c) +
                              (slice + (int64_t)row0 * args.ldc + col0) * kEsz;
#pragma unroll
                for (int k = 0; k < 32 / kRowsPer; ++k) {
                  const int r = k * kRowsPer + lane / kPieces, p = lane % kPieces;
                  const int phys = OUT == kOutBf16 ? (p ^ ((r >> 1) & 3)) : (p ^ (r & 7));
                  int4 val = *reinterpret_cast<const int4*>(stg + r * (kPieces * 16) + phys * 16);
                  if constexpr (OUT == kOutBf16 && !PEERS) {
                    // residual + bf16(x W^T + b), the residual piece of the same (row, piece)
                    if (args.residual && row0 + r < args.m) {
                      const __nv_bfloat16* re = reinterpret_cast<const __nv_bfloat16*>(&rres[k]);
                      __nv_bfloat16* vb = reinterpret_cast<__nv_bfloat16*>(&val);
#pragma unroll
                      for (int e = 0; e < 8; ++e)
                        vb[e] = __float2bfloat16_rn(__bfloat162float(re[e]) + __bfloat162float(vb[e]));
                    }
                  }
                  if (row0 + r < args.m) {
                    int4* dst = reinterpret_cast<int4*>(cb + ((int64_t)r * args.ldc) * kEsz + p * 16);
                    if constexpr ((XB_L2_HINTS & 1) != 0 && !PEERS) __stcs(dst, val);
                    else *dst = val;
                  }
                }
              }
              __syncwarp();  // staging free for the next chunk
              continue;
            }
          }
        }
        if (row >= args.m || col0 >= args.n) continue;
        if constexpr (OUT != kOutI32) {
          if (args.bias) {  // bias indexed by the output feature: the row of W
            const __nv_bfloat16* bp = static_cast<const __nv_bfloat16*>(args.bias);
            if constexpr (TRANS) {
              const float bv = __bfloat162float(bp[row]);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + bv);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (col0 + j < args.n) v[j] = __float_as_uint(__uint_as_float(v[j]) + __bfloat162float(bp[col0 + j]));
            }
          }
        }
        if constexpr (TRANS) {
          // lanes hold consecutive rows: each j is one coalesced row segment of C
          if constexpr (OUT == kOutBf16) {
            __nv_bfloat16* cp = static_cast<__nv_bfloat16*>(args.c) + slice + row;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < args.n) cp[(int64_t)(col0 + j) * args.ldc] = __float2bfloat16_rn(__uint_as_float(v[j]));
          } else {
            uint32_t* cp = static_cast<uint32_t*>(args.c) + slice + row;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < args.n) cp[(int64_t)(col0 + j) * args.ldc] = v[j];
          }
        } else {
        if constexpr (OUT == kOutBf16) {
          if (args.act == 1) {
#pragma unroll
            for (int jj = 0; jj < 32; ++jj)
              v[jj] = __float_as_uint(gelu_tanh_bf16path(__bfloat162float(__float2bfloat16_rn(__uint_as_float(v[jj])))));
          }
        }
        if constexpr (OUT == kOutBf16 && !TRANS && !PEERS) {
          if (args.residual && row < args.m) {  // y = residual + bf16(x W^T + b), as a linear then an add round
            const __nv_bfloat16* rp = static_cast<const __nv_bfloat16*>(args.residual) + (int64_t)row * args.ldr + col0;
            if (col0 + 32 <= args.n && ((reinterpret_cast<uintptr_t>(rp) & 15) == 0)) {
#pragma unroll
              for (int j = 0; j < 32; j += 8) {
                const int4 raw = __ldg(reinterpret_cast<const int4*>(rp + j));
                const __nv_bfloat16* re = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
                for (int e = 0; e < 8; ++e)
                  v[j + e] = __float_as_uint(__bfloat162float(re[e]) +
                                             __bfloat162float(__float2bfloat16_rn(__uint_as_float(v[j + e]))));
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (col0 + j < args.n)
                  v[j] = __float_as_uint(__bfloat162float(rp[j]) +
                                         __bfloat162float(__float2bfloat16_rn(__uint_as_float(v[j]))));
            }
          }
        }
#pragma unroll 1
         for (int pe = 0; pe < (PEERS ? args.world : 1); ++pe) {
          void* cbase = PEERS ? args.peers[pe] : args.c;
          if constexpr (OUT == kOutBf16) {
          __nv_bfloat16* cp = static_cast<__nv_bfloat16*>(cbase) + slice + (int64_t)row * args.ldc + col0;
          if (col0 + 32 <= args.n && ((reinterpret_cast<uintptr_t>(cp) & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              __nv_bfloat162 h[4];
#pragma unroll
              for (int e = 0; e < 4; ++e)
                h[e] = __floats2bfloat162_rn(__uint_as_float(v[j + 2 * e]), __uint_as_float(v[j + 2 * e + 1]));
              *reinterpret_cast<int4*>(cp + j) = *reinterpret_cast<int4*>(h);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < args.n) cp[j] = __float2bfloat16_rn(__uint_as_float(v[j]));
          }
          } else {
          uint32_t* cp = static_cast<uint32_t*>(cbase) + slice + (int64_t)row * args.ldc + col0;
          if (col0 + 32 <= args.n && ((reinterpret_cast<uintptr_t>(cp) & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<uint4*>(cp + j) = make_uint4(v[j], v[j + 1], v[j + 2], v[j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < args.n) cp[j] = v[j];
          }
          }
         }
        }
      }
      tc_fence_before();
      if constexpr (PAIR) mbar_arrive_cluster(mapa_u32(smem_u32(&tempty_bar[buf]), 0));
      else mbar_arrive(&tempty_bar[buf]);
    }
    if constexpr (!PEERS && OUT != kOutSwiglu && (TRANS || OUT != kOutBf16)) {
      if (args.c_tma && lane == 0) bulk_wait_all();  // every TMA store of C has completed
      __syncwarp();
    }
  }

  if constexpr (PEERS) __threadfence_system();  // this thread's peer stores, before the CTA is counted done
  __syncthreads();
  if constexpr (PEERS) {
    // Every CTA counts itself once, aborted or not, so the counter always
    // returns to zero at the end of a call; an aborted CTA also adds 2^32.
    // The last CTA signals the peers only when no CTA aborted: a peer then
    // times out in its wait (an error status) instead of reading a C whose
    // tiles were partly skipped.
    if (threadIdx.x == 0) {
      uint64_t* done = args.signals[args.rank] + args.world;
      const unsigned long long add = abort_flag ? (1ull << 32) + 1ull : 1ull;
      const unsigned long long prev = atomicAdd(reinterpret_cast<unsigned long long*>(done), add);
      if ((prev & 0xffffffffull) == gridDim.x - 1) {  // last CTA of the grid
        if ((prev >> 32) == 0 && !abort_flag) {  // every tile of this rank has landed everywhere
          __threadfence_system();
          for (int pe = 0; pe < args.world; ++pe)
            if (pe != args.rank) red_release_sys_add(args.signals[pe] + args.rank, 1ull);
        }
        *done = 0;  // no CTA of this grid touches it again; ready for the next call
      }
    }
  }
  if constexpr (PAIR) {
    // Neither CTA leaves while the other may still read its shared memory
    // (MMA operands), signal its barriers or write its TMEM.
    tc_fence_before();
    cluster_sync();
  }
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc2(tmem_base, C::TMEM_COLS);
    else tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// Y[m, n] = [residual[m, n] +] round(sum_s part[s, m, n] + bias[n]): the
// split-K reduction of the small-M linear, in a fixed order (deterministic),
// fused with the bias and the residual add that follow o_proj / down_proj.
// With bf16 output the linear result is rounded to bf16 before the residual
// add, as two separate bf16 operations would round it.
template <bool OUT_BF16>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ part, int splits, int64_t M,
                                                            int64_t N, const __nv_bfloat16* __restrict__ bias,
                                                            const __nv_bfloat16* __restrict__ residual, int64_t ldr,
                                                            void* __restrict__ y, int64_t ldy) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / N, n = i - m * N;
    float acc = 0.0f;
    for (int s2 = 0; s2 < splits; ++s2) acc += part[(int64_t)s2 * total + i];
    if (bias) acc += __bfloat162float(bias[n]);
    if constexpr (OUT_BF16) {
      float r = __bfloat162float(__float2bfloat16_rn(acc));
      if (residual) r = __bfloat162float(residual[m * ldr + n]) + r;
      static_cast<__nv_bfloat16*>(y)[m * ldy + n] = __float2bfloat16_rn(r);
    } else {
      if (residual) acc += __bfloat162float(residual[m * ldr + n]);
      static_cast<float*>(y)[m * ldy + n] = acc;
    }
  }
}

// Vectorised forms of the two reductions below (4 consecutive outputs per
// thread, one CTA row per token, no 64-bit division); the summation order is
// the same, so results are identical.  Used when every pointer and pitch is
// aligned for 16-byte partial loads and 8-byte bf16 accesses.
__device__ __forceinline__ void add4(float4& a, const float4 b) {
  a.x += b.x;
  a.y += b.y;
  a.z += b.z;
  a.w += b.w;
}
__device__ __forceinline__ float4 ld_bf16x4(const __nv_bfloat16* p) {
  const uint2 raw = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
  return make_float4(__low2float(h[0]), __high2float(h[0]), __low2float(h[1]), __high2float(h[1]));
}
__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
// acc += p[s * slice] for s = 1 .. splits-1, in that order, four loads in
// flight at a time (the order of the additions is the plain loop's).
__device__ __forceinline__ void sum_splits4(float4& acc, const float* p, int splits, int64_t slice) {
  int s2 = 1;
  for (; s2 + 8 <= splits; s2 += 8) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = __ldcg(reinterpret_cast<const float4*>(p + (s2 + u) * slice));
#pragma unroll
    for (int u = 0; u < 8; ++u) add4(acc, v[u]);
  }
  for (; s2 + 4 <= splits; s2 += 4) {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(p + s2 * slice));
    const float4 b = __ldcg(reinterpret_cast<const float4*>(p + (s2 + 1) * slice));
    const float4 c = __ldcg(reinterpret_cast<const float4*>(p + (s2 + 2) * slice));
    const float4 d = __ldcg(reinterpret_cast<const float4*>(p + (s2 + 3) * slice));
    add4(acc, a);
    add4(acc, b);
    add4(acc, c);
    add4(acc, d);
  }
  for (; s2 < splits; ++s2) add4(acc, __ldcg(reinterpret_cast<const float4*>(p + s2 * slice)));
}
__device__ __forceinline__ float sum_splits1(const float* p, int splits, int64_t slice) {
  float acc = __ldcg(p);
  int s2 = 1;
  for (; s2 + 8 <= splits; s2 += 8) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = __ldcg(p + (s2 + u) * slice);
#pragma unroll
    for (int u = 0; u < 8; ++u) acc += v[u];
  }
  for (; s2 + 4 <= splits; s2 += 4) {
    const float a = __ldcg(p + s2 * slice), b = __ldcg(p + (s2 + 1) * slice);
    const float c = __ldcg(p + (s2 + 2) * slice), d = __ldcg(p + (s2 + 3) * slice);
    acc += a;
    acc += b;
    acc += c;
    acc += d;
  }
  for (; s2 < splits; ++s2) acc += __ldcg(p + s2 * slice);
  return acc;
}
__device__ __forceinline__ void st_bf16x4(__nv_bfloat16* p, float a, float b, float c, float d) {
  __nv_bfloat162 h[2] = {__floats2bfloat162_rn(a, b), __floats2bfloat162_rn(c, d)};
  *reinterpret_cast<uint2*>(p) = *reinterpret_cast<uint2*>(h);
}

template <bool OUT_BF16, bool GELU = false>
__global__ void __launch_bounds__(256) splitk_reduce4_kernel(const float* __restrict__ part, int splits, int M, int N,
                                                             const __nv_bfloat16* __restrict__ bias,
                                                             const __nv_bfloat16* __restrict__ residual, int64_t ldr,
                                                             void* __restrict__ y, int64_t ldy) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.y;
  const int n = (blockIdx.x * 256 + threadIdx.x) * 4;
  if (n >= N) return;
  const int64_t slice = (int64_t)M * N;
  const float* p = part + (int64_t)m * N + n;
  float4 acc = __ldcg(reinterpret_cast<const float4*>(p));
  sum_splits4(acc, p, splits, slice);
  if (bias) add4(acc, ld_bf16x4(bias + n));
  if constexpr (OUT_BF16) {
    float4 r = make_float4(rbf(acc.x), rbf(acc.y), rbf(acc.z), rbf(acc.w));
    if constexpr (GELU)
      r = make_float4(gelu_tanh_bf16path(r.x), gelu_tanh_bf16path(r.y), gelu_tanh_bf16path(r.z),
                      gelu_tanh_bf16path(r.w));
    if (residual) {
      const float4 q = ld_bf16x4(residual + m * ldr + n);
      r = make_float4(q.x + r.x, q.y + r.y, q.z + r.z, q.w + r.w);
    }
    st_bf16x4(static_cast<__nv_bfloat16*>(y) + m * ldy + n, r.x, r.y, r.z, r.w);
  } else {
    if (residual) add4(acc, ld_bf16x4(residual + m * ldr + n));
    *reinterpret_cast<float4*>(static_cast<float*>(y) + m * ldy + n) = acc;
  }
}

// IL: W interleaves 64-row blocks of gate and up rows (the kOutSwiglu layout);
// otherwise gate rows [0, n_out) are stacked over up rows [n_out, 2 n_out).
template <bool IL>
__global__ void __launch_bounds__(256) splitk_swiglu4_kernel(const float* __restrict__ part, int splits, int M,
                                                             int n_out, __nv_bfloat16* __restrict__ y, int64_t ldy) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.y;
  const int f = (blockIdx.x * 256 + threadIdx.x) * 4;
  if (f >= n_out) return;
  const int64_t slice = (int64_t)M * 2 * n_out;
  const int gcol = IL ? ((f >> 6) << 7) + (f & 63) : f;
  const int ucol = gcol + (IL ? 64 : n_out);
  const float* pg = part + (int64_t)m * 2 * n_out + gcol;
  const float* pu = part + (int64_t)m * 2 * n_out + ucol;
  float4 g = __ldcg(reinterpret_cast<const float4*>(pg));
  float4 u = __ldcg(reinterpret_cast<const float4*>(pu));
  sum_splits4(g, pg, splits, slice);
  sum_splits4(u, pu, splits, slice);
  auto sw = [](float gg, float uu) { return __fmul_rn(silu_bf16path(rbf(gg)), rbf(uu)); };
  st_bf16x4(y + m * ldy + f, sw(g.x, u.x), sw(g.y, u.y), sw(g.z, u.z), sw(g.w, u.w));
}

// ---- decode-step fusions of the split-K reduction -------------------------
//
// reduce_rope_kv_kernel: the fused QKV projection of one decode token per CTA
// (M = batch rows, one position), finished in place of the reduce + RoPE/KV
// kernels: v = bf16(sum_s part + bias) exactly as the reduction rounds it,
// then the rotate-half RoPE of the query and key heads (skipped without
// tables) with the same fp32 products and sums as the stand-alone RoPE
// kernel, written to q [B, H, 1, D] and the K / V caches at `pos`.
__global__ void __launch_bounds__(1024) reduce_rope_kv_kernel(const float* __restrict__ part, int splits, int M,
                                                              int N, const __nv_bfloat16* __restrict__ bias,
                                                              const float* __restrict__ cos_t,
                                                              const float* __restrict__ sin_t,
                                                              __nv_bfloat16* __restrict__ q_out,
                                                              __nv_bfloat16* __restrict__ k_cache,
                                                              __nv_bfloat16* __restrict__ v_cache, int H, int KVH,
                                                              int D, int smax, int pos) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x;
  const int half = D / 2;
  const int slots = H + 2 * KVH;
  const int64_t slice = (int64_t)M * N;
  const float* pr = part + (int64_t)m * N;
  // blockIdx.y splits the token's (head slot, pair) items over gridDim.y CTAs
  const int per = (slots * half + gridDim.y - 1) / gridDim.y;
  const int j0 = blockIdx.y * per, j1 = min(slots * half, j0 + per);
  for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) {
    const int slot = j / half;
    const int i = j - slot * half;
    const int f0 = slot * D + i, f1 = f0 + half;
    float a0 = sum_splits1(pr + f0, splits, slice), a1 = sum_splits1(pr + f1, splits, slice);
    if (bias) {
      a0 += __bfloat162float(bias[f0]);
      a1 += __bfloat162float(bias[f1]);
    }
    const __nv_bfloat16 x0b = __float2bfloat16_rn(a0), x1b = __float2bfloat16_rn(a1);
    if (slot >= H + KVH) {
      __nv_bfloat16* dst = v_cache + (((int64_t)m * KVH + (slot - H - KVH)) * smax + pos) * D;
      dst[i] = x0b;
      dst[i + half] = x1b;
      continue;
    }
    __nv_bfloat16* dst = slot < H ? q_out + ((int64_t)m * H + slot) * D
                                  : k_cache + (((int64_t)m * KVH + (slot - H)) * smax + pos) * D;
    if (!cos_t) {
      dst[i] = x0b;
      dst[i + half] = x1b;
      continue;
    }
    const float x0 = __bfloat162float(x0b), x1 = __bfloat162float(x1b);
    const float* cr = cos_t + (int64_t)pos * D;
    const float* sr = sin_t + (int64_t)pos * D;
    dst[i] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(x0, cr[i]), __fmul_rn(-x1, sr[i])));
    dst[i + half] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(x1, cr[i + half]), __fmul_rn(x0, sr[i + half])));
  }
}

// reduce_residual_norm_kernel: one CTA per row m of a decode step.
//   y  = bf16(residual + bf16(sum_s part + bias))      (the residual stream)
//   yn = bf16(norm(y))                                  (input of the next linear)
// NORM 0: y * rsqrt(mean(y^2) + eps) * w (RMSNorm); NORM 1: (y - mean) *
// rsqrt(var + eps) * w + b (LayerNorm), both in fp32 over the bf16 y.  Each
// thread keeps its 4-column groups in registers (N <= 4096).
template <int NORM>
__global__ void __launch_bounds__(256) reduce_residual_norm_kernel(
    const float* __restrict__ part, int splits, int M, int N, const __nv_bfloat16* __restrict__ bias,
    const __nv_bfloat16* __restrict__ residual, int64_t ldr, __nv_bfloat16* __restrict__ y, int64_t ldy,
    __nv_bfloat16* __restrict__ yn, int64_t ldn, const __nv_bfloat16* __restrict__ nw,
    const __nv_bfloat16* __restrict__ nb, float eps) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[8];
  __shared__ float bcast;
  const int m = blockIdx.x, tid = threadIdx.x;
  const int64_t slice = (int64_t)M * N;
  float4 v[4];
  float s1 = 0.0f;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int n = (tid + 256 * g) * 4;
    v[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (n >= N) continue;
    const float* p = part + (int64_t)m * N + n;
    float4 acc = __ldcg(reinterpret_cast<const float4*>(p));
    sum_splits4(acc, p, splits, slice);
    if (bias) add4(acc, ld_bf16x4(bias + n));
    const float4 r = ld_bf16x4(residual + m * ldr + n);
    const float4 o = make_float4(rbf(r.x + rbf(acc.x)), rbf(r.y + rbf(acc.y)), rbf(r.z + rbf(acc.z)),
                                 rbf(r.w + rbf(acc.w)));
    st_bf16x4(y + m * ldy + n, o.x, o.y, o.z, o.w);
    v[g] = o;
    s1 += NORM == 0 ? (o.x * o.x + o.y * o.y) + (o.z * o.z + o.w * o.w) : (o.x + o.y) + (o.z + o.w);
  }
  auto block_sum = [&](float x) {
#pragma unroll
    for (int o_ = 16; o_ > 0; o_ >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o_);
    if ((tid & 31) == 0) red[tid >> 5] = x;
    __syncthreads();
    if (tid == 0) {
      float t = 0.0f;
#pragma unroll
      for (int w = 0; w < 8; ++w) t += red[w];
      bcast = t;
    }
    __syncthreads();
    const float r = bcast;
    __syncthreads();
    return r;
  };
  const float inv_n = 1.0f / (float)N;
  float mean = 0.0f, rstd;
  if constexpr (NORM == 0) {
    rstd = __frsqrt_rn(block_sum(s1) * inv_n + eps);
  } else {
    mean = block_sum(s1) * inv_n;
    float s2 = 0.0f;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int n = (tid + 256 * g) * 4;
      if (n >= N) continue;
      const float a = v[g].x - mean, b = v[g].y - mean, c = v[g].z - mean, d = v[g].w - mean;
      s2 += (a * a + b * b) + (c * c + d * d);
    }
    rstd = __frsqrt_rn(block_sum(s2) * inv_n + eps);
  }
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int n = (tid + 256 * g) * 4;
    if (n >= N) continue;
    const float4 w4 = ld_bf16x4(nw + n);
    if constexpr (NORM == 0) {
      st_bf16x4(yn + m * ldn + n, __fmul_rn(__fmul_rn(v[g].x, rstd), w4.x), __fmul_rn(__fmul_rn(v[g].y, rstd), w4.y),
                __fmul_rn(__fmul_rn(v[g].z, rstd), w4.z), __fmul_rn(__fmul_rn(v[g].w, rstd), w4.w));
    } else {
      const float4 b4 = nb ? ld_bf16x4(nb + n) : make_float4(0.f, 0.f, 0.f, 0.f);
      st_bf16x4(yn + m * ldn + n, (v[g].x - mean) * rstd * w4.x + b4.x, (v[g].y - mean) * rstd * w4.y + b4.y,
                (v[g].z - mean) * rstd * w4.z + b4.z, (v[g].w - mean) * rstd * w4.w + b4.w);
    }
  }
}

// The decode MLP: W stacks the gate rows [0, n_out) over the up rows
// [n_out, 2 n_out); y[m, f] = bf16(silu(bf16(g)) * bf16(u)) with g, u the
// split-K sums of gate row f and up row f -- the same roundings as a gate
// linear, an up linear and the silu*up kernel run one after another.
__global__ void __launch_bounds__(256) splitk_swiglu_kernel(const float* __restrict__ part, int splits, int64_t M,
                                                            int64_t n_out, __nv_bfloat16* __restrict__ y,
                                                            int64_t ldy) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = M * n_out;
  const int64_t slice = M * 2 * n_out;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / n_out, f = i - m * n_out;
    float g = 0.0f, u = 0.0f;
    for (int s2 = 0; s2 < splits; ++s2) {
      g += part[(int64_t)s2 * slice + m * 2 * n_out + f];
      u += part[(int64_t)s2 * slice + m * 2 * n_out + n_out + f];
    }
    g = __bfloat162float(__float2bfloat16_rn(g));
    u = __bfloat162float(__float2bfloat16_rn(u));
    y[m * ldy + f] = __float2bfloat16_rn(__fmul_rn(silu_bf16path(g), u));
  }
}

// Split count for the small-M linear: enough (weight-row tile, K slice)
// work units to cover the SMs (a slice may be a single 64-wide K block).
int small_m_splits(int64_t N, int64_t K) {
  const int64_t tiles = (N + 127) / 128;
  const int64_t kblocks = (K + 63) / 64;
  int sms = 148;
  sm_count(&sms);
  int64_t want = (sms + tiles - 1) / tiles;
  const int64_t cap = kblocks;
  if (want > cap) want = cap;
  if (want < 1) want = 1;
  const int64_t kps = (kblocks + want - 1) / want;
  return (int)((kblocks + kps - 1) / kps);
}

// int16 -> (high s8, low u8) limb planes, each [rows, cols] with leading dim ldp.
__global__ void split_i16_kernel(const int16_t* __restrict__ src, int64_t rows, int64_t cols, int64_t lds,
                                 int8_t* __restrict__ hi, uint8_t* __restrict__ lo, int64_t ldp) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    const int16_t v = src[r * lds + c];
    hi[r * ldp + c] = (int8_t)(v >> 8);
    lo[r * ldp + c] = (uint8_t)(v & 0xFF);
  }
}

// int16 [K, N] (pitch lds) -> (high s8, low u8) limb planes stored transposed,
// [N, ldp] (K-major, the B operand layout of the limb GEMM); K <= k < ldp is
// zero.  32 x 32 tiles through shared memory, 32 x 8 threads.
__global__ void __launch_bounds__(256) split_i16_t_kernel(const int16_t* __restrict__ src, int64_t K, int64_t N,
                                                          int64_t lds, int8_t* __restrict__ hi,
                                                          uint8_t* __restrict__ lo, int64_t ldp) {
  pdl_wait();
  pdl_trigger();
  __shared__ int16_t tile[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t n0 = (int64_t)blockIdx.x * 32, k0 = (int64_t)blockIdx.y * 32;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t k = k0 + ty + 8 * i, n = n0 + tx;
    tile[ty + 8 * i][tx] = (k < K && n < N) ? src[k * lds + n] : (int16_t)0;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t n = n0 + ty + 8 * i, k = k0 + tx;
    if (n < N && k < ldp) {
      const int16_t v = tile[tx][ty + 8 * i];
      hi[n * ldp + k] = (int8_t)(v >> 8);
      lo[n * ldp + k] = (uint8_t)(v & 0xFF);
    }
  }
}

// ------------------------------------------------------------------------- host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder(char* err, size_t errlen) {
  static EncodeTiledFn fn = nullptr;
  if (fn) return fn;
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p) {
    set_err(err, errlen, "cuTensorMapEncodeTiled unavailable: %s", cudaGetErrorString(e));
    return nullptr;
  }
  fn = reinterpret_cast<EncodeTiledFn>(p);
  return fn;
}

// 2-D tiled map over a row-major matrix [outer, inner] with 128-byte swizzle.
int make_map(CUtensorMap* map, const void* ptr, CUtensorMapDataType dt, int esz, uint64_t inner, uint64_t outer,
             uint64_t ld_elems, uint32_t box_inner, uint32_t box_outer, char* err, size_t errlen) {
  EncodeTiledFn enc = encoder(err, errlen);
  if (!enc) return XB_ERR_CUDA;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_elems * (uint64_t)esz};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_err(err, errlen, "cuTensorMapEncodeTiled failed (%d) for a %llux%llu operand", (int)r,
            (unsigned long long)outer, (unsigned long long)inner);
    return XB_ERR_CUDA;
  }
  return XB_OK;
}

// 3-D map [outer2][outer1][inner] (strides in elements), box {bi, bo, 1},
// no swizzle: plain row-major staging tiles.
int make_map_3d(CUtensorMap* map, const void* ptr, CUtensorMapDataType dt, int esz, uint64_t inner, uint64_t outer1,
                uint64_t outer2, uint64_t ld1, uint64_t ld2, uint32_t box_inner, uint32_t box_outer, char* err,
                size_t errlen) {
  EncodeTiledFn enc = encoder(err, errlen);
  if (!enc) return XB_ERR_CUDA;
  cuuint64_t dims[3] = {inner, outer1, outer2};
  cuuint64_t strides[2] = {ld1 * (uint64_t)esz, ld2 * (uint64_t)esz};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_err(err, errlen, "cuTensorMapEncodeTiled failed (%d) for a %llux%llux%llu output", (int)r,
            (unsigned long long)outer2, (unsigned long long)outer1, (unsigned long long)inner);
    return XB_ERR_CUDA;
  }
  return XB_OK;
}

bool tma_ok(const void* p, int64_t ld, int esz) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && (ld * esz) % 16 == 0;
}

struct Operands {
  const void* a[2];
  const void* b[2];
  int64_t lda, ldb;
};

struct PeerArgs {
  int world = 1, rank = 0;
  void* peers[8] = {nullptr};
  uint64_t* signals[8] = {nullptr};
  uint64_t epoch = 0, timeout_ns = 0;
};

// Launch with clusters of two CTAs (and programmatic dependent launch when enabled).
template <typename... KArgs, typename... Args2>
cudaError_t launch_pairs(void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t s,
                         Args2... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  prefer_max_smem(reinterpret_cast<const void*>(kernel));
  launch_counter().fetch_add(1, std::memory_order_relaxed);
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

bool lines_enabled();
bool epi8_enabled();

template <int KIND, bool B_KMAJOR, int OUT, int BN_ = 0, bool TRANS = false, bool PEERS = false, bool PAIR = false,
          int EPI = 4>
int launch(const Operands& op, void* c, const void* bias, int64_t M, int64_t N, int64_t K, int64_t ldc,
           cudaStream_t s, const char* what, char* err, size_t errlen, int splits = 1, int64_t split_stride = 0,
           const PeerArgs* pa = nullptr, const void* residual = nullptr, int64_t ldr = 0, int act = 0,
           const Args* qkv = nullptr) {
  using Cf = Cfg<KIND, B_KMAJOR, BN_, PAIR>;
  const CUtensorMapDataType dt = KIND == kBf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  Maps maps;
  memset(&maps, 0, sizeof(maps));
  for (int p = 0; p < Cf::PLANES; ++p) {
    int rc = make_map(&maps.a[p], op.a[p], dt, Cf::ESZ, K, M, op.lda, Cf::BK, Cf::BM, err, errlen);
    if (rc) return rc;
    rc = B_KMAJOR ? make_map(&maps.b[p], op.b[p], dt, Cf::ESZ, K, N, op.ldb, Cf::BK, Cf::BN_CTA, err, errlen)
                  : make_map(&maps.b[p], op.b[p], dt, Cf::ESZ, N, K, op.ldb, Cf::B_BOX_N, Cf::BK, err, errlen);
    if (rc) return rc;
  }
  Args args;
  memset(&args, 0, sizeof(args));
  if (qkv) args = *qkv;  // kOutQkv destinations
  args.c = c;
  args.bias = bias;
  args.residual = residual;
  args.ldr = ldr;
  args.act = act;
  args.ldc = ldc;
  args.m = (int)M;
  args.n = (int)N;
  args.k = (int)K;
  args.tiles_m = (int)((M + Cf::TILE_M - 1) / Cf::TILE_M);
  args.tiles_n = (int)((N + Cf::BN - 1) / Cf::BN);
  args.kblocks = (int)((K + Cf::BK - 1) / Cf::BK);
  if (splits < 1) splits = 1;
  if (splits > args.kblocks) splits = args.kblocks;
  args.kps = (args.kblocks + splits - 1) / splits;
  args.splits = (args.kblocks + args.kps - 1) / args.kps;  // every slice gets at least one K block
  args.split_stride = split_stride;
  args.num_tiles = args.tiles_m * args.tiles_n * args.splits;
  args.world = pa ? pa->world : 1;
  args.rank = pa ? pa->rank : 0;
  for (int i = 0; i < 8; ++i) {
    args.peers[i] = pa ? pa->peers[i] : nullptr;
    args.signals[i] = pa ? pa->signals[i] : nullptr;
  }
  args.epoch = pa ? pa->epoch : 0;
  args.peer_timeout_ns = pa ? pa->timeout_ns : 0;
  // 4-byte outputs of whole-tile GEMMs leave through the TMA-store epilogue
  // when C meets the TMA alignment rules.
  // Transposed (small-M) outputs too, through [tokens][features] staging tiles.
  constexpr bool kStaged =
      !PEERS && OUT != kOutSwiglu && OUT != kOutArgmax && OUT != kOutQkv && (TRANS || OUT != kOutBf16);
  constexpr bool kLines = !TRANS && (PEERS || OUT == kOutBf16);  // whole-line staged stores
  static_assert(OUT != kOutQkv || !TRANS, "the fused QKV epilogue takes row-major tiles");
  constexpr int kSmem = Cf::SMEM + ((kStaged || kLines || OUT == kOutArgmax || OUT == kOutQkv) ? kEpiStageBytes : 0);
  static_assert(4 * 32 * 33 * 4 + 4 * 64 * 8 <= kEpiStageBytes, "argmax staging fits");
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
  args.c_tma = 0;
  if constexpr (kStaged && !TRANS) {
    if (args.splits == 1 && tma_ok(c, ldc, 4)) {
      int rc = make_map(&maps.c, c, OUT == kOutI32 ? CU_TENSOR_MAP_DATA_TYPE_INT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                        4, N, M, ldc, 32, 32, err, errlen);
      if (rc) return rc;
      args.c_tma = 1;
    }
  }
  if constexpr (kStaged && TRANS) {
    const int esz = OUT == kOutBf16 ? 2 : 4;
    if (tma_ok(c, ldc, esz) && (args.splits == 1 || (split_stride * esz) % 16 == 0)) {
      int rc = make_map_3d(&maps.c, c, OUT == kOutBf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                           esz, (uint64_t)M, (uint64_t)N, (uint64_t)args.splits, (uint64_t)ldc,
                           (uint64_t)(args.splits == 1 ? ldc * N : split_stride), 32, 32, err, errlen);
      if (rc) return rc;
      args.c_tma = 1;
    }
  }
  if constexpr (kLines) {  // whole-line stores need 16-byte aligned rows everywhere
    const int esz = OUT == kOutBf16 ? 2 : 4;
    bool ok = (ldc * esz) % 16 == 0 && args.splits == 1 && (PEERS || lines_enabled());
    if (PEERS) {
      for (int i = 0; i < args.world; ++i) ok = ok && (reinterpret_cast<uintptr_t>(args.peers[i]) & 15) == 0;
    } else {
      ok = ok && (reinterpret_cast<uintptr_t>(c) & 15) == 0;
    }
    // the whole-line epilogue reads the residual in 16-byte pieces: its base
    // and row pitch must be 16-byte aligned too (else the per-row path, which
    // checks every segment, runs)
    if (residual) ok = ok && (reinterpret_cast<uintptr_t>(residual) & 15) == 0 && (ldr * 2) % 16 == 0;
    args.c_tma = ok ? 1 : 0;
  }
  auto kernel = gemm_kernel<KIND, B_KMAJOR, OUT, BN_, TRANS, PEERS, PAIR, EPI>;
  constexpr unsigned kBlock = 64 + 32 * EPI;
  // shared-memory limit and (pairs) the resident cluster count, once per device
  int max_clusters = 0;
  {
    cudaError_t e = once_per_device(reinterpret_cast<const void*>(kernel), kOnceSmem, [&](int* v) {
      cudaError_t r = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
      if (r == cudaSuccess && PAIR) {
        // resident pairs: the persistent grid is sized to what runs at once
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2);
        cfg.blockDim = dim3(kBlock);
        cfg.dynamicSmemBytes = kSmem;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = 2;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        r = cudaOccupancyMaxActiveClusters(v, kernel, &cfg);
        if (r == cudaSuccess && *v < 1) r = cudaErrorInvalidConfiguration;
      }
      return r;
    }, &max_clusters);
    if (e != cudaSuccess) {
      set_err(err, errlen, "%s: kernel setup: %s", what, cudaGetErrorString(e));
      return XB_ERR_CUDA;
    }
  }
  int sms = 148;
  sm_count(&sms);
  if constexpr (PAIR) {
    const int clusters = args.num_tiles < max_clusters ? args.num_tiles : max_clusters;
    cudaError_t e = launch_pairs(kernel, 2 * clusters, kBlock, kSmem, s, maps, args);
    if (e != cudaSuccess) {
      set_err(err, errlen, "%s: %s", what, cudaGetErrorString(e));
      return XB_ERR_CUDA;
    }
  } else {
    const int grid = args.num_tiles < sms ? args.num_tiles : sms;
    launch_k(kernel, grid, kBlock, kSmem, s, maps, args);
  }
  return check_launch(what, err, errlen);
}

// CTA pairs for products with at least two 128-row blocks; XB_GEMM_PAIRS=0
// in the environment selects the single-CTA kernel everywhere.
// XB_GEMM_LINES=0 in the environment keeps per-thread row stores (A/B timing).
bool lines_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("XB_GEMM_LINES");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// Epilogue warps of bf16-output / fused-QKV CTA-pair tiles: eight (two per
// TMEM lane quarter); XB_GEMM_EPI=4 in the environment selects four.
bool epi8_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("XB_GEMM_EPI");
    on = (v && atoi(v) == 4) ? 0 : 1;
  }
  return on == 1;
}

bool use_pairs(int64_t M) {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("XB_GEMM_PAIRS");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1 && M >= 256;
}

int check_common(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                 int64_t ldc, bool b_kmajor, const char* what, char* err, size_t errlen) {
  if (M < 0 || N < 0 || K < 0) { set_err(err, errlen, "%s: negative shape", what); return XB_ERR_INVALID; }
  if (M > 0x7fffff00LL || N > 0x7fffff00LL || K > 0x7fffff00LL) {
    set_err(err, errlen, "%s: dimension too large", what);
    return XB_ERR_UNSUPPORTED;
  }
  if (M == 0 || N == 0) return 1;  // nothing to do
  if (!C || (K > 0 && (!A || !B))) { set_err(err, errlen, "%s: null pointer", what); return XB_ERR_INVALID; }
  if (lda < K || ldc < N || ldb < (b_kmajor ? K : N)) {
    set_err(err, errlen, "%s: leading dimension smaller than the row (lda=%lld ldb=%lld ldc=%lld)", what,
            (long long)lda, (long long)ldb, (long long)ldc);
    return XB_ERR_INVALID;
  }
  return 0;
}

int zero_fill(void* C, int64_t M, int64_t N, int64_t ldc, int esz, cudaStream_t s, const char* what, char* err,
              size_t errlen) {
  cudaError_t e = cudaMemset2DAsync(C, ldc * esz, 0, N * esz, M, s);
  if (e != cudaSuccess) { set_err(err, errlen, "%s: %s", what, cudaGetErrorString(e)); return XB_ERR_CUDA; }
  return XB_OK;
}

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Workspace layout for the int16 limb planes (each plane 256-byte aligned,
// rows padded to a multiple of 16 bytes for TMA).
struct LimbLayout {
  int64_t lda_p, ldb_p;
  size_t a_plane, b_plane, total;
};
LimbLayout limb_layout(int64_t M, int64_t N, int64_t K) {
  LimbLayout L;
  // both limb operands K-major: A planes [M, lda_p], B planes transposed [N, ldb_p]
  L.lda_p = (int64_t)round_up((size_t)(K > 0 ? K : 1), 16);
  L.ldb_p = L.lda_p;
  L.a_plane = round_up((size_t)(M > 0 ? M : 1) * L.lda_p, 256);
  L.b_plane = round_up((size_t)(N > 0 ? N : 1) * L.ldb_p, 256);
  L.total = 2 * L.a_plane + 2 * L.b_plane;
  return L;
}

int split_launch(const int16_t* src, int64_t rows, int64_t cols, int64_t lds, int8_t* hi, uint8_t* lo, int64_t ldp,
                 cudaStream_t s) {
  const int64_t total = rows * cols;
  int64_t grid = (total + 255) / 256;
  if (grid > 148 * 32) grid = 148 * 32;
  if (grid < 1) grid = 1;
  launch_k(split_i16_kernel, (unsigned)grid, 256, 0, s, src, rows, cols, lds, hi, lo, ldp);
  return 0;
}

int run_i16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
            int64_t ldc, void* ws, size_t ws_bytes, cudaStream_t s, const char* what, char* err, size_t errlen) {
  int rc = check_common(A, B, C, M, N, K, lda, ldb, ldc, false, what, err, errlen);
  if (rc) return rc < 0 ? rc : XB_OK;
  if (K == 0) return zero_fill(C, M, N, ldc, 4, s, what, err, errlen);
  const LimbLayout L = limb_layout(M, N, K);
  if (!ws || ws_bytes < L.total) {
    set_err(err, errlen, "%s: workspace of %zu bytes given, %zu needed", what, ws_bytes, L.total);
    return XB_ERR_INVALID;
  }
  if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0) {
    set_err(err, errlen, "%s: workspace must be 256-byte aligned", what);
    return XB_ERR_INVALID;
  }
  if ((reinterpret_cast<uintptr_t>(C) & 3) != 0) {
    set_err(err, errlen, "%s: C must be 4-byte aligned", what);
    return XB_ERR_INVALID;
  }
  uint8_t* w = static_cast<uint8_t*>(ws);
  int8_t* ahi = reinterpret_cast<int8_t*>(w);
  uint8_t* alo = w + L.a_plane;
  int8_t* bhi = reinterpret_cast<int8_t*>(w + 2 * L.a_plane);
  uint8_t* blo = w + 2 * L.a_plane + L.b_plane;
  split_launch(static_cast<const int16_t*>(A), M, K, lda, ahi, alo, L.lda_p, s);
  {
    const dim3 grid((unsigned)((N + 31) / 32), (unsigned)((L.ldb_p + 31) / 32));
    if (grid.y > 65535) {
      set_err(err, errlen, "%s: K too large for the limb transpose grid", what);
      return XB_ERR_UNSUPPORTED;
    }
    launch_k(split_i16_t_kernel, grid, 256, 0, s, static_cast<const int16_t*>(B), K, N, ldb, bhi, blo, L.ldb_p);
  }
  rc = check_launch(what, err, errlen);
  if (rc) return rc;
  Operands op{{ahi, alo}, {bhi, blo}, L.lda_p, L.ldb_p};
  if (use_pairs(M)) return launch<kInt16Limbs, true, kOutI32, 0, false, false, true>(op, C, nullptr, M, N, K, ldc, s,
                                                                                       what, err, errlen);
  return launch<kInt16Limbs, true, kOutI32>(op, C, nullptr, M, N, K, ldc, s, what, err, errlen);
}

}  // namespace gemm
}  // namespace xb

using namespace xb::gemm;
using xb::set_err;
using xb::check_launch;
using xb::launch_k;

extern "C" int xb_matmul_i8(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                            int64_t ldb, int64_t ldc, void* stream, char* err, size_t errlen) {
  const char* what = "xb_matmul_i8";
  cudaStream_t s = (cudaStream_t)stream;
  int rc = check_common(A, B, C, M, N, K, lda, ldb, ldc, false, what, err, errlen);
  if (rc) return rc < 0 ? rc : XB_OK;
  if (K == 0) return zero_fill(C, M, N, ldc, 4, s, what, err, errlen);
  if (!tma_ok(A, lda, 1) || !tma_ok(B, ldb, 1)) {
    set_err(err, errlen, "%s: A/B must be 16-byte aligned with row pitches a multiple of 16 bytes", what);
    return XB_ERR_UNSUPPORTED;
  }
  Operands op{{A, nullptr}, {B, nullptr}, lda, ldb};
  if (use_pairs(M)) return launch<kInt8, false, kOutI32, 0, false, false, true>(op, C, nullptr, M, N, K, ldc, s, what, err, errlen);
  return launch<kInt8, false, kOutI32>(op, C, nullptr, M, N, K, ldc, s, what, err, errlen);
}

extern "C" int xb_linear_i8(const void* X, const void* W, void* Y, int64_t M, int64_t N, int64_t K, int64_t ldx,
                            int64_t ldw, int64_t ldy, void* stream, char* err, size_t errlen) {
  const char* what = "xb_linear_i8";
  cudaStream_t s = (cudaStream_t)stream;
  int rc = check_common(X, W, Y, M, N, K, ldx, ldw, ldy, true, what, err, errlen);
  if (rc) return rc < 0 ? rc : XB_OK;
  if (K == 0) return zero_fill(Y, M, N, ldy, 4, s, what, err, errlen);
  if (!tma_ok(X, ldx, 1) || !tma_ok(W, ldw, 1)) {
    set_err(err, errlen, "%s: X/W must be 16-byte aligned with row pitches a multiple of 16 bytes", what);
    return XB_ERR_UNSUPPORTED;
  }
  Operands op{{X, nullptr}, {W, nullptr}, ldx, ldw};
  if (use_pairs(M)) return launch<kInt8, true, kOutI32, 0, false, false, true>(op, Y, nullptr, M, N, K, ldy, s, what, err, errlen);
  return launch<kInt8, true, kOutI32>(op, Y, nullptr, M, N, K, ldy, s, what, err, errlen);
}

extern "C" int xb_matmul_i16_workspace_size(int64_t M, int64_t N, int64_t K, size_t* bytes, char* err,
                                            size_t errlen) {
  if (!bytes || M < 0 || N < 0 || K < 0) {
    set_err(err, errlen, "xb_matmul_i16_workspace_size: bad arguments");
    return XB_ERR_INVALID;
  }
  *bytes = limb_layout(M, N, K).total;
  return XB_OK;
}

extern "C" int xb_matmul_i16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                             int64_t ldb, int64_t ldc, void* workspace, size_t workspace_bytes, void* stream,
                             char* err, size_t errlen) {
  return run_i16(A, B, C, M, N, K, lda, ldb, ldc, workspace, workspace_bytes, (cudaStream_t)stream, "xb_matmul_i16",
                 err, errlen);
}

// ---------------------------------------------------------------------------
// int16 GEMM for callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc at all: plugins whose host framework
// owns every device allocation through its own pool (memory taken behind its
// back breaks its accounting and limits), and latency-bound paths where a
// cudaMalloc may synchronise the device and stall.  xb_matmul_i16 needs a
// caller-provided workspace for its int8
// limb planes; this variant instead keeps them in a fixed-size array compiled
// into the library (XB_I16_NOALLOC_SCRATCH_BYTES per GPU, resident on every
// GPU that loads this module until the process exits).  The caller still
// passes A, B and C.
//
// In host code the array's name is only a host-side stand-in, so its device
// address is looked up once per device with cudaGetSymbolAddress, with that
// device current, on the first call made on it.  That first call must
// therefore come before any stream capture on the device.  All calls share the
// one array: calls whose GPU work overlaps (two streams, or two host threads)
// race on it.  The split kernel rewrites every limb byte the GEMM reads before
// it reads them, so nothing has to start at zero, and stale contents from an
// earlier call are never used.
static __device__ __align__(256) uint8_t g_i16_noalloc_scratch[XB_I16_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {nullptr};
}  // namespace

extern "C" int xb_matmul_i16_noalloc(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                                     int64_t lda, int64_t ldb, int64_t ldc, void* stream, char* err, size_t errlen) {
  const char* what = "xb_matmul_i16_noalloc";
  if (M < 0 || N < 0 || K < 0) {
    set_err(err, errlen, "%s: negative shape", what);
    return XB_ERR_INVALID;
  }
  const size_t need = limb_layout(M, N, K).total;
  if (need > (size_t)XB_I16_NOALLOC_SCRATCH_BYTES) {
    set_err(err, errlen,
            "%s: an %lldx%lldx%lld product needs %zu bytes of limb scratch, more than the built-in %zu bytes; "
            "use xb_matmul_i16 with a workspace",
            what, (long long)M, (long long)N, (long long)K, need, (size_t)XB_I16_NOALLOC_SCRATCH_BYTES);
    return XB_ERR_UNSUPPORTED;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    set_err(err, errlen, "%s: no usable current device (%s)", what, cudaGetErrorString(e));
    return XB_ERR_CUDA;
  }
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_i16_noalloc_scratch);
      if (e != cudaSuccess || !p) {
        set_err(err, errlen, "%s: cudaGetSymbolAddress of the scratch array failed on device %d: %s", what, dev,
                cudaGetErrorString(e));
        return XB_ERR_CUDA;
      }
      g_noalloc_ptr[dev] = p;
    }
    scratch = g_noalloc_ptr[dev];
  }
  return run_i16(A, B, C, M, N, K, lda, ldb, ldc, scratch, (size_t)XB_I16_NOALLOC_SCRATCH_BYTES,
                 (cudaStream_t)stream, what, err, errlen);
}

extern "C" int xb_matmul_bf16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                              int64_t ldb, int64_t ldc, int out_dtype, void* stream, char* err, size_t errlen) {
  const char* what = "xb_matmul_bf16";
  cudaStream_t s = (cudaStream_t)stream;
  if (out_dtype != XB_DT_F32 && out_dtype != XB_DT_BF16) {
    set_err(err, errlen, "%s: out_dtype must be f32 or bf16", what);
    return XB_ERR_UNSUPPORTED;
  }
  int rc = check_common(A, B, C, M, N, K, lda, ldb, ldc, false, what, err, errlen);
  if (rc) return rc < 0 ? rc : XB_OK;
  const int osz = out_dtype == XB_DT_F32 ? 4 : 2;
  if (K == 0) return zero_fill(C, M, N, ldc, osz, s, what, err, errlen);
  if (!tma_ok(A, lda, 2) || !tma_ok(B, ldb, 2)) {
    set_err(err, errlen, "%s: A/B must be 16-byte aligned with row pitches a multiple of 16 bytes", what);
    return XB_ERR_UNSUPPORTED;
  }
  Operands op{{A, nullptr}, {B, nullptr}, lda, ldb};
  if (use_pairs(M)) {
    if (out_dtype == XB_DT_F32)
      return launch<kBf16, false, kOutF32, 0, false, false, true>(op, C, nullptr, M, N, K, ldc, s, what, err, errlen);
    if (epi8_enabled())
      return launch<kBf16, false, kOutBf16, 0, false, false, true, 8>(op, C, nullptr, M, N, K, ldc, s, what, err,
                                                                      errlen);
    return launch<kBf16, false, kOutBf16, 0, false, false, true>(op, C, nullptr, M, N, K, ldc, s, what, err, errlen);
  }
  if (out_dtype == XB_DT_F32) return launch<kBf16, false, kOutF32>(op, C, nullptr, M, N, K, ldc, s, what, err, errlen);
  return launch<kBf16, false, kOutBf16>(op, C, nullptr, M, N, K, ldc, s, what, err, errlen);
}

extern "C" int xb_linear_bf16(const void* X, const void* W, const void* bias, void* Y, int64_t M, int64_t N,
                              int64_t K, int64_t ldx, int64_t ldw, int64_t ldy, int out_dtype, void* stream,
                              char* err, size_t errlen) {
  const char* what = "xb_linear_bf16";
  cudaStream_t s = (cudaStream_t)stream;
  if (out_dtype != XB_DT_F32 && out_dtype != XB_DT_BF16) {
    set_err(err, errlen, "%s: out_dtype must be f32 or bf16", what);
    return XB_ERR_UNSUPPORTED;
  }
  int rc = check_common(X, W, Y, M, N, K, ldx, ldw, ldy, true, what, err, errlen);
  if (rc) return rc < 0 ? rc : XB_OK;
  if (K == 0) {
    set_err(err, errlen, "%s: K must be positive", what);
    return XB_ERR_INVALID;
  }
  if (!tma_ok(X, ldx, 2) || !tma_ok(W, ldw, 2)) {
    set_err(err, errlen, "%s: X/W must be 16-byte aligned with row pitches a multiple of 16 bytes", what);
    return XB_ERR_UNSUPPORTED;
  }
  Operands op{{X, nullptr}, {W, nullptr}, ldx, ldw};
  if (use_pairs(M)) {
    if (out_dtype == XB_DT_F32)
      return launch<kBf16, true, kOutF32, 0, false, false, true>(op, Y, bias, M, N, K, ldy, s, what, err, errlen);
    if (epi8_enabled())
      return launch<kBf16, true, kOutBf16, 0, false, false, true, 8>(op, Y, bias, M, N, K, ldy, s, what, err, errlen);
    return launch<kBf16, true, kOutBf16, 0, false, false, true>(op, Y, bias, M, N, K, ldy, s, what, err, errlen);
  }
  if (out_dtype == XB_DT_F32) return launch<kBf16, true, kOutF32>(op, Y, bias, M, N, K, ldy, s, what, err, errlen);
  return launch<kBf16, true, kOutBf16>(op, Y, bias, M, N, K, ldy, s, what, err, errlen);
}

namespace xb {
namespace gemm {

// ---- decode linears: split-K over a thread-block cluster, finished in place ----
//
// Y = X W^T for the few tokens of a decode step (M <= 64), with the work that
// follows the linear in the same launch.  A cluster of S CTAs owns one
// 128-row block of W (128 output features x all tokens); CTA r of the
// cluster multiplies K blocks [r kps, (r+1) kps) into a 128 x 64 fp32 TMEM
// accumulator (tcgen05, swap-AB: weight rows are the MMA's M, tokens its N).
// CTA q of the cluster owns tokens [q pt, (q+1) pt), pt = ceil(64 / S): every
// CTA pushes the rows of its partial that belong to CTA q into q's receive
// buffer over distributed shared memory (16-byte stores), one cluster
// barrier publishes them, and each CTA sums the S partials of its tokens from
// its own shared memory in rank order (deterministic), then applies the
// finisher:
//   kFinStore     y = bf16(acc + bias), optionally the tanh GELU on that value
//   kFinRopeKv    qkv = bf16(acc + bias), rotate-half RoPE of the query / key
//                 heads, written to q [B, H, D] and the K / V caches at `pos`
//   kFinSwiglu    W interleaves 64-row blocks of gate and up rows; y =
//                 bf16(silu(bf16(g)) * bf16(u)) for the block's 64 features
//   kFinResidual  y = bf16(residual + bf16(acc + bias)), plus per (128-row
//                 block, token) statistics of y for the norm that follows:
//                 the sum of squares (RMSNorm) or the block mean and sum of
//                 squared deviations (LayerNorm, combined later with Chan's
//                 parallel formula)
// The partial sums never leave the chip (no split-K workspace, no second
// kernel), and no CTA touches another's shared memory after the barrier, so
// none waits for its peers before it exits.  A pending norm of X (XNORM) is
// applied as X is loaded: the consumer combines the producer's block
// statistics per token (fixed order) and, while the weight tiles stream, the
// epilogue warps rewrite each X tile in shared memory as bf16(norm(x)) before
// the MMA reads it -- so a residual add, the norm after it and the next
// linear take two launches, not four.  Everything that does not depend on the
// previous kernel (weight tiles of the first ring slots, norm weights, bias)
// is requested before the programmatic-launch wait.
enum Fin { kFinStore = 0, kFinRopeKv = 1, kFinSwiglu = 2, kFinResidual = 3 };

constexpr int kDecBM = 128;                   // weight rows per cluster (TMEM lanes)
constexpr int kDecBN = 64;                    // tokens (MMA N)
constexpr int kDecBK = 64;                    // K elements per ring slot (128 bytes of bf16)
constexpr int kDecA = kDecBM * 128;           // weight tile bytes per slot
constexpr int kDecStage = kDecA + kDecBN * 128;
constexpr int kDecRedBytes = kDecBN * kDecBM * 4;  // this CTA's fp32 partial [token][row], over the ring
constexpr int kDecMaxCluster = 16;            // CTAs per cluster at most (above 8: non-portable cluster size)
// receive buffer [source rank][owned token][row] fp32: S * ceil(64 / S) <= 72 token rows
constexpr int kDecRecvBytes = 72 * kDecBM * 4;

struct DecMaps {
  CUtensorMap w;  // W [N, K] K-major, 64 x 128 boxes
  CUtensorMap x;  // X [M, K] K-major, 64 x 64 boxes (rows past M read as zero)
};

struct DecArgs {
  int m, n, k;                 // tokens, weight rows, K
  int kblocks, kps, splits;    // K blocks of 64, per CTA, CTAs per cluster
  // pending norm of X (XNORM): block statistics [ceil(K / 128)][64] of its rows
  const float2* xstats;
  const __nv_bfloat16* xnw;
  const __nv_bfloat16* xnb;    // LayerNorm bias or null
  float xeps;
  int xkind;                   // 0 RMSNorm, 1 LayerNorm
  const __nv_bfloat16* bias;   // [n] or null
  __nv_bfloat16* y;            // Store / Swiglu / Residual output
  int64_t ldy;
  int act;                     // Store: 1 = tanh GELU
  const __nv_bfloat16* residual;
  int64_t ldr;
  float2* stats;               // Residual: statistics of y [ceil(n / 128)][64], or null
  int stats_kind;              // 0 RMSNorm (sum of squares), 1 LayerNorm (mean, M2)
  const float* cos_t;          // RopeKv: [positions, D] tables or null (no rotation)
  const float* sin_t;
  __nv_bfloat16* q_out;        // [B, H, D]
  __nv_bfloat16* k_cache;      // [B, KVH, smax, D]
  __nv_bfloat16* v_cache;
  int H, KVH, D, smax, pos;
};

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o_ = 16; o_ > 0; o_ >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o_);
  return x;
}

__device__ __forceinline__ void st_dsmem_f4(uint32_t addr, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

// ---- decode finishers, shared by the one-launch decode linear and the decode chain
//
// After the split-K reduction, CTA `rank` of a cluster owns tokens [tok0,
// tok0 + ntok) of a 128-row weight block (row0 = 128 * blk); its receive
// buffer rv holds, per source rank jr < S, the partial rows [jr * pt + tl][128]
// as float4.  The four epilogue warps (warps 2..5) finish the block.

constexpr int kDecPre = 4;  // residual rows requested ahead, per epilogue thread

// Loads a finisher requests long before it uses them.  Volatile asm keeps
// them where they are written (ahead of the barrier waits) instead of letting
// the compiler sink them next to their use on the critical path.
__device__ __forceinline__ uint2 ld_early_cg_u2(const void* p) {
  uint2 v;  // L2 load: residual rows may have been written earlier in the same launch
  asm volatile("ld.global.cg.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ float4 ld_early_nc_f4(const float* p) {
  float4 v;  // read-only tables
  asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ float4 bf16x4_to_f4(uint2 raw) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
  return make_float4(__low2float(h[0]), __high2float(h[0]), __low2float(h[1]), __high2float(h[1]));
}
__device__ __forceinline__ float4 ld_bf16x4_cg(const __nv_bfloat16* p) { return bf16x4_to_f4(ld_early_cg_u2(p)); }

// Bias and RoPE rows an epilogue thread uses for every unit of one block.
struct DecConsts {
  float4 pb0, pb1, pc0, pc1, ps0, ps1;
};

template <int FIN>
__device__ __forceinline__ DecConsts dec_consts(const DecArgs& args, int row0, int lane) {
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  DecConsts k{z4, z4, z4, z4, z4, z4};
  if constexpr (FIN == kFinStore || FIN == kFinResidual) {
    const int n = row0 + lane * 4;
    if (args.bias && n < args.n) k.pb0 = ld_bf16x4_cg(args.bias + n);
  } else if constexpr (FIN == kFinRopeKv) {
    const int half = args.D >> 1, p = (lane & 15) * 4, hd = p / half, i = p - hd * half;
    const int f0 = row0 + hd * args.D + i, slot = (row0 + hd * args.D) / args.D;
    if (slot < args.H + 2 * args.KVH) {
      if (args.bias) {
        k.pb0 = ld_bf16x4_cg(args.bias + f0);
        k.pb1 = ld_bf16x4_cg(args.bias + f0 + half);
      }
      if (args.cos_t && slot < args.H + args.KVH) {
        const float* cr = args.cos_t + (int64_t)args.pos * args.D;
        const float* sr = args.sin_t + (int64_t)args.pos * args.D;
        k.pc0 = ld_early_nc_f4(cr + i);
        k.pc1 = ld_early_nc_f4(cr + i + half);
        k.ps0 = ld_early_nc_f4(sr + i);
        k.ps1 = ld_early_nc_f4(sr + i + half);
      }
    }
  }
  return k;
}

// Residual rows of the first kDecPre owned tokens of this epilogue warp.
template <int FIN>
__device__ __forceinline__ void dec_rpre(const DecArgs& args, int ntok, int tok0, int row0, int warp, int lane,
                                         float4 (&rpre)[kDecPre]) {
  if constexpr (FIN == kFinResidual) {
#pragma unroll
    for (int u = 0; u < kDecPre; ++u) {
      const int tl = (warp - 2) + 4 * u, n = row0 + lane * 4;
      rpre[u] = tl < ntok && n < args.n ? ld_bf16x4_cg(args.residual + (tok0 + tl) * args.ldr + n)
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

template <int FIN>
__device__ __forceinline__ void dec_finish(const DecArgs& args, const float4* rv, int S, int pt, int ntok, int tok0,
                                           int row0, int blk, int warp, int lane, const DecConsts& kc,
                                           const float4 (&rpre)[kDecPre]) {
  const int e = (warp - 2) * 32 + lane;  // 0 .. 127
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  constexpr int kSlot = kDecBM / 4;  // float4 per token row of the receive buffer
  // acc[u] = sum of the S partials of (owned token tl[u], rows c[u]..c[u]+3), rank
  // order; the loads of up to four units are issued together
  auto gather4 = [&](const int (&tl)[4], const int (&c)[4], const bool (&ok)[4], float4 (&acc)[4]) {
#pragma unroll
    for (int u = 0; u < 4; ++u) acc[u] = ok[u] ? rv[tl[u] * kSlot + (c[u] >> 2)] : z4;
#pragma unroll
    for (int jr = 1; jr < kDecMaxCluster; ++jr) {
      if (jr < S) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = ok[u] ? rv[(jr * pt + tl[u]) * kSlot + (c[u] >> 2)] : z4;
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (ok[u]) add4(acc[u], v[u]);
      }
    }
  };
  if constexpr (FIN == kFinStore) {
    // units (owned token, 4-row group): thread e takes units e + 128 k, all with rows c
    const int c = (e & 31) * 4, n = row0 + c;
    for (int u0 = e; u0 < ntok * 32; u0 += 4 * 128) {
      int tl[4], cc[4];
      bool ok[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        tl[u] = (u0 + 128 * u) >> 5;
        cc[u] = c;
        ok[u] = u0 + 128 * u < ntok * 32 && n < args.n;
      }
      float4 acc[4];
      gather4(tl, cc, ok, acc);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (!ok[u]) continue;
        add4(acc[u], kc.pb0);
        float4 o = make_float4(rbf(acc[u].x), rbf(acc[u].y), rbf(acc[u].z), rbf(acc[u].w));
        if (args.act == 1)
          o = make_float4(gelu_tanh_bf16path(o.x), gelu_tanh_bf16path(o.y), gelu_tanh_bf16path(o.z),
                          gelu_tanh_bf16path(o.w));
        st_bf16x4(args.y + (tok0 + tl[u]) * args.ldy + n, o.x, o.y, o.z, o.w);
      }
    }
  } else if constexpr (FIN == kFinResidual) {
    // warp per owned token (tokens w, w + 4, ... of the epilogue warp w), lane =
    // 4-row group: the block statistics of a token row reduce within the warp;
    // four tokens at a time, their loads and reductions interleaved
    const int c = lane * 4, n = row0 + c;
    const bool valid = n < args.n;
    const float cnt = (float)min(kDecBM, args.n - row0);
    for (int ub = 0; (warp - 2) + 16 * ub < ntok; ++ub) {
      int tl[4], cc[4];
      bool ok[4], live[4];
      float4 r[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        tl[u] = (warp - 2) + 4 * (4 * ub + u);
        cc[u] = c;
        live[u] = tl[u] < ntok;  // warp-uniform
        ok[u] = live[u] && valid;
        r[u] = ub == 0 ? rpre[u]
                       : (ok[u] ? ld_bf16x4_cg(args.residual + (tok0 + tl[u]) * args.ldr + n) : z4);
      }
      float4 acc[4], o[4];
      gather4(tl, cc, ok, acc);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        o[u] = z4;
        if (!ok[u]) continue;
        add4(acc[u], kc.pb0);
        o[u] = make_float4(rbf(r[u].x + rbf(acc[u].x)), rbf(r[u].y + rbf(acc[u].y)), rbf(r[u].z + rbf(acc[u].z)),
                           rbf(r[u].w + rbf(acc[u].w)));
        st_bf16x4(args.y + (tok0 + tl[u]) * args.ldy + n, o[u].x, o[u].y, o[u].z, o[u].w);
      }
      if (args.stats) {
        float s1[4], s2[4], sh[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float4 v = o[u];
          if (args.stats_kind == 0) {
            sh[u] = 0.0f;
            s1[u] = (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
            s2[u] = 0.0f;
          } else {
            // shifted sums (shift: the block's first value) give the block mean
            // and the sum of squared deviations in one pass
            sh[u] = __shfl_sync(0xffffffffu, v.x, 0);
            const float a = v.x - sh[u], b = v.y - sh[u], cz = v.z - sh[u], d = v.w - sh[u];
            s1[u] = valid ? (a + b) + (cz + d) : 0.0f;
            s2[u] = valid ? (a * a + b * b) + (cz * cz + d * d) : 0.0f;
          }
        }
#pragma unroll
        for (int o_ = 16; o_ > 0; o_ >>= 1) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            s1[u] += __shfl_xor_sync(0xffffffffu, s1[u], o_);
            s2[u] += __shfl_xor_sync(0xffffffffu, s2[u], o_);
          }
        }
        if (lane == 0) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (!live[u]) continue;
            args.stats[blk * kDecBN + tok0 + tl[u]] =
                args.stats_kind == 0 ? make_float2(s1[u], 0.0f)
                                     : make_float2(sh[u] + s1[u] / cnt, fmaxf(s2[u] - s1[u] * s1[u] / cnt, 0.0f));
          }
        }
      }
    }
  } else if constexpr (FIN == kFinSwiglu) {
    // rows [0, 64) gate and [64, 128) up of features blk*64 .. blk*64+63;
    // units (owned token, 4 features): thread e takes units e + 128 k
    const int c = (e & 15) * 4;
    for (int u0 = e; u0 < ntok * 16; u0 += 2 * 128) {
      int tl[4], cc[4];
      bool ok[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {  // (gate, up) of two units
        tl[u] = (u0 + 128 * (u >> 1)) >> 4;
        cc[u] = c + 64 * (u & 1);
        ok[u] = u0 + 128 * (u >> 1) < ntok * 16;
      }
      float4 acc[4];
      gather4(tl, cc, ok, acc);
      auto sw = [](float gg, float uu) { return __fmul_rn(silu_bf16path(rbf(gg)), rbf(uu)); };
#pragma unroll
      for (int u = 0; u < 4; u += 2) {
        if (!ok[u]) continue;
        const float4 g = acc[u], up = acc[u + 1];
        st_bf16x4(args.y + (tok0 + tl[u]) * args.ldy + blk * 64 + c, sw(g.x, up.x), sw(g.y, up.y), sw(g.z, up.z),
                  sw(g.w, up.w));
      }
    }
  } else {
    // kFinRopeKv: units (owned token, 4 consecutive rotation pairs of one head);
    // thread e takes units e + 128 k, all with the same pairs
    const int D = args.D, half = D >> 1;
    const int p = (e & 15) * 4;  // first pair index within the block
    const int hd = p / half, i = p - hd * half;
    const int c0 = hd * D + i;   // row of the first element, within the block
    const int slot = (row0 + hd * D) / D;
    if (slot < args.H + 2 * args.KVH) {
      for (int u0 = e; u0 < ntok * 16; u0 += 2 * 128) {
        int tl[4], cc[4];
        bool ok[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {  // (first, second half) of two units
          tl[u] = (u0 + 128 * (u >> 1)) >> 4;
          cc[u] = c0 + half * (u & 1);
          ok[u] = u0 + 128 * (u >> 1) < ntok * 16;
        }
        float4 acc[4];
        gather4(tl, cc, ok, acc);
#pragma unroll
        for (int u = 0; u < 4; u += 2) {
          if (!ok[u]) continue;
          const int t = tok0 + tl[u];
          float4 a0 = acc[u], a1 = acc[u + 1];
          add4(a0, kc.pb0);
          add4(a1, kc.pb1);
          const float x0[4] = {rbf(a0.x), rbf(a0.y), rbf(a0.z), rbf(a0.w)};
          const float x1[4] = {rbf(a1.x), rbf(a1.y), rbf(a1.z), rbf(a1.w)};
          __nv_bfloat16* dst;
          if (slot < args.H)
            dst = args.q_out + ((int64_t)t * args.H + slot) * D;
          else if (slot < args.H + args.KVH)
            dst = args.k_cache + (((int64_t)t * args.KVH + (slot - args.H)) * args.smax + args.pos) * D;
          else
            dst = args.v_cache + (((int64_t)t * args.KVH + (slot - args.H - args.KVH)) * args.smax + args.pos) * D;
          float o0[4], o1[4];
          if (slot >= args.H + args.KVH || !args.cos_t) {
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              o0[jj] = x0[jj];
              o1[jj] = x1[jj];
            }
          } else {
            const float c0v[4] = {kc.pc0.x, kc.pc0.y, kc.pc0.z, kc.pc0.w};
            const float c1v[4] = {kc.pc1.x, kc.pc1.y, kc.pc1.z, kc.pc1.w};
            const float s0v[4] = {kc.ps0.x, kc.ps0.y, kc.ps0.z, kc.ps0.w};
            const float s1v[4] = {kc.ps1.x, kc.ps1.y, kc.ps1.z, kc.ps1.w};
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              o0[jj] = __fadd_rn(__fmul_rn(x0[jj], c0v[jj]), __fmul_rn(-x1[jj], s0v[jj]));
              o1[jj] = __fadd_rn(__fmul_rn(x1[jj], c1v[jj]), __fmul_rn(x0[jj], s1v[jj]));
            }
          }
          st_bf16x4(dst + i, o0[0], o0[1], o0[2], o0[3]);
          st_bf16x4(dst + i + half, o1[0], o1[1], o1[2], o1[3]);
        }
      }
    }
  }
}

template <int FIN, int STAGES, bool XNORM>
__global__ void __launch_bounds__(192, 1) decode_linear_kernel(const __grid_constant__ DecMaps maps,
                                                               const DecArgs args) {
  static_assert(STAGES * kDecStage >= kDecRedBytes, "the partial fits over the ring");
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t xready_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t tfull_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;
  __shared__ float s_mean[kDecBN], s_rstd[kDecBN];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t base_u32 = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - smem_u32(smem_raw));
  float* recv = reinterpret_cast<float*>(smem + STAGES * kDecStage);  // not the ring: peers write it any time
  const int S = args.splits;
  const int rank = (int)cluster_ctarank();
  const int blk = (int)blockIdx.x / S;  // 128-row block of W
  const int kb0 = rank * args.kps;
  const int nkb = min(kb0 + args.kps, args.kblocks) - kb0;  // >= 1 (host picks S so)
  const int pt = (kDecBN + S - 1) / S;                       // tokens owned per CTA
  const int tok0 = rank * pt, ntok = max(0, min(args.m, tok0 + pt) - tok0);
  const int row0 = blk * kDecBM;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&xready_bar[s], 128);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&tfull_bar, 1);
    abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&maps.w);
    prefetch_tmap(&maps.x);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, kDecBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  if (warp == 1) {
    pdl_wait();
    pdl_trigger();
  }
  auto fail = [&]() {
    atomicExch(&g_gemm_status, XB_ERR_TIMEOUT);
    abort_flag = 1;
  };

  // Residual finisher: warp w of the epilogue takes owned tokens w, w + 4, ...;
  // their residual rows are requested while the MMAs run.
  float4 rpre[kDecPre];
  // Finisher constants (bias, RoPE table rows), requested before the
  // programmatic-launch wait: every finisher unit of a thread uses the same rows.
  DecConsts kc = {};
  if (warp >= 2) kc = dec_consts<FIN>(args, row0, lane);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const int npre = min(STAGES, nkb);
      for (int i = 0; i < npre; ++i) {
        mbar_arrive_expect_tx(&full_bar[i], kDecStage);
        tma_load_2d(smem + i * kDecStage, &maps.w, &full_bar[i], (kb0 + i) * kDecBK, row0);
      }
      pdl_wait();  // X is written by the previous kernel
      pdl_trigger();
      for (int i = 0; i < npre; ++i)
        tma_load_2d(smem + i * kDecStage + kDecA, &maps.x, &full_bar[i], (kb0 + i) * kDecBK, 0);
      int issued = npre;
      for (int i = npre; i < nkb; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(&empty_bar[s], ((i / STAGES) & 1) ^ 1, kWaitLimit, &abort_flag)) {
          fail();
          break;
        }
        mbar_arrive_expect_tx(&full_bar[s], kDecStage);
        tma_load_2d(smem + s * kDecStage, &maps.w, &full_bar[s], (kb0 + i) * kDecBK, row0);
        tma_load_2d(smem + s * kDecStage + kDecA, &maps.x, &full_bar[s], (kb0 + i) * kDecBK, 0);
        issued = i + 1;
      }
      // every load issued must have landed before the ring is reused or the CTA
      // exits (also after an abort; one time limit for all of them)
      uint64_t deadline = 0;
      for (int i = issued > STAGES ? issued - STAGES : 0; i < issued; ++i)
        if (!mbar_wait_deadline(&full_bar[i % STAGES], (i / STAGES) & 1, &deadline, kWaitLimit)) fail();
    } else {
      pdl_wait();
      pdl_trigger();
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int done = 0;
      for (int i = 0; i < nkb; ++i, ++done) {
        const int s = i % STAGES;
        uint64_t* ready = XNORM ? &xready_bar[s] : &full_bar[s];
        if (!mbar_wait(ready, (i / STAGES) & 1, kWaitLimit, &abort_flag)) {
          fail();
          break;
        }
        tc_fence_after();
        const uint32_t st = base_u32 + s * kDecStage;
#pragma unroll
        for (int ks = 0; ks < kDecBK / 16; ++ks)
          mma_f16(tmem_base, umma_desc_sw128(st + ks * 32, 16, 1024), umma_desc_sw128(st + kDecA + ks * 32, 16, 1024),
                  umma_idesc(1, 1, 1, 0, 0, kDecBM, kDecBN), (i > 0 || ks > 0) ? 1u : 0u);
        tc_commit(&empty_bar[s]);
      }
      if (done > 0) {
        tc_commit(&tfull_bar);  // the accumulator is final once these MMAs complete
        // The issuing thread itself sees them complete (whatever the abort
        // flag says) before the TMEM can be released after the cluster barrier.
        volatile int never = 0;
        if (!mbar_wait(&tfull_bar, 0, kWaitLimit, &never)) fail();
      }
    }
    __syncwarp();
  } else {
    const int e = threadIdx.x - 64;  // 0 .. 127
    if constexpr (XNORM) {
      // ---------------------------------------------------------- X tiles -> bf16(norm(X))
      // Thread e rewrites the 16-byte chunks (token (e >> 3) + 16 jj, K
      // elements 8 (e & 7) .. + 7) of every slot: one norm-weight vector per
      // slot, the first requested before the wait (the weights are constant).
      const int j = e & 7;
      auto ld_w = [&](int i, uint4& w, uint4& b) {
        const int k0 = (kb0 + i) * kDecBK + j * 8;
        w = make_uint4(0u, 0u, 0u, 0u);
        b = make_uint4(0u, 0u, 0u, 0u);
        if (i < nkb && k0 < args.k) {
          w = __ldg(reinterpret_cast<const uint4*>(args.xnw + k0));
          if (args.xkind == 1 && args.xnb) b = __ldg(reinterpret_cast<const uint4*>(args.xnb + k0));
        }
      };
      uint4 wn, bn;
      ld_w(0, wn, bn);
      pdl_wait();
      pdl_trigger();
      if (e < kDecBN) {  // per-token mean / rstd from the producer's block statistics, in block order
        const int t = e;
        float mean = 0.0f, rstd = 0.0f;
        if (t < args.m) {
          const int nb = (args.k + kDecBM - 1) / kDecBM;
          float na = 0.0f, ma = 0.0f, acc = 0.0f;
          for (int b0 = 0; b0 < nb; b0 += 8) {  // eight loads in flight, then the fixed-order combine
            float2 st[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
              st[u] = b0 + u < nb ? __ldcg(&args.xstats[(b0 + u) * kDecBN + t]) : make_float2(0.f, 0.f);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              if (b0 + u >= nb) break;
              if (args.xkind == 0) {
                acc += st[u].x;
              } else {  // Chan et al.: merge (n_b, mean_b, M2_b) into the running (n, mean, M2)
                const float nbk = (float)min(kDecBM, args.k - (b0 + u) * kDecBM);
                const float n = na + nbk, delta = st[u].x - ma;
                ma += delta * (nbk / n);
                acc += st[u].y + delta * delta * (na * nbk / n);
                na = n;
              }
            }
          }
          mean = args.xkind == 0 ? 0.0f : ma;
          rstd = __frsqrt_rn(acc / (float)args.k + args.xeps);
        }
        s_mean[t] = mean;
        s_rstd[t] = rstd;
      }
      epi_bar();
      for (int i = 0; i < nkb; ++i) {
        const int s = i % STAGES;
        const uint4 wraw = wn, braw = bn;
        ld_w(i + 1, wn, bn);  // the next slot's weights, while this one is rewritten
        if (!mbar_wait(&full_bar[s], (i / STAGES) & 1, kWaitLimit, &abort_flag)) {
          fail();
          break;
        }
        uint8_t* xs = smem + s * kDecStage + kDecA;  // [64 tokens][128 bytes], 128-byte swizzle
        const __nv_bfloat162* wh = reinterpret_cast<const __nv_bfloat162*>(&wraw);
        const __nv_bfloat162* bh = reinterpret_cast<const __nv_bfloat162*>(&braw);
        if ((kb0 + i) * kDecBK + j * 8 < args.k) {  // past K: zero-filled, stays zero
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int r = (e >> 3) + 16 * jj;
            uint4* p = reinterpret_cast<uint4*>(xs + r * 128 + ((j ^ (r & 7)) << 4));
            uint4 raw = *p;
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
            const float mean = s_mean[r], rstd = s_rstd[r];
            if (args.xkind == 0) {
#pragma unroll
              for (int q2 = 0; q2 < 4; ++q2)
                h[q2] = __floats2bfloat162_rn(__fmul_rn(__fmul_rn(__low2float(h[q2]), rstd), __low2float(wh[q2])),
                                              __fmul_rn(__fmul_rn(__high2float(h[q2]), rstd), __high2float(wh[q2])));
            } else {
#pragma unroll
              for (int q2 = 0; q2 < 4; ++q2)
                h[q2] = __floats2bfloat162_rn(
                    (__low2float(h[q2]) - mean) * rstd * __low2float(wh[q2]) + __low2float(bh[q2]),
                    (__high2float(h[q2]) - mean) * rstd * __high2float(wh[q2]) + __high2float(bh[q2]));
            }
            *p = raw;
          }
        }
        fence_proxy_async_smem();  // these writes, before the MMA's (async-proxy) reads
        mbar_arrive(&xready_bar[s]);
      }
    } else {
      pdl_wait();
      pdl_trigger();
    }
    dec_rpre<FIN>(args, ntok, tok0, row0, warp, lane, rpre);
    // ------------------------------------------------------------ accumulator -> owners
    const int q = warp & 3;  // TMEM lane quarter this warp may read
    const bool got = mbar_wait(&tfull_bar, 0, kWaitLimit, &abort_flag);
    if (!got) fail();
    float* red = reinterpret_cast<float*>(smem);  // [token][row], over the ring (this CTA's MMAs are done)
    if (got) {
      tc_fence_after();
      fence_proxy_async_smem();
      const int row = q * 32 + lane;
#pragma unroll
      for (int h = 0; h < kDecBN / 32; ++h) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + h * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) red[(h * 32 + jj) * kDecBM + row] = __uint_as_float(v[jj]);
      }
    }
    tc_fence_before();
    epi_bar();
    if (got) {
      // token t's row of the partial -> slot `rank` of its owner's receive
      // buffer; thread e sends rows (e & 31) * 4 .. + 3 of tokens e / 32 + 4 k
      // (t grows by 4 < pt per step, so the owner advances at most by one)
      const uint32_t recv0 = smem_u32(recv);
      int t = e >> 5, owner = t / pt, tl = t - owner * pt;
      uint32_t peer = mapa_u32(recv0, (uint32_t)owner);
      for (; t < args.m; t += 4, tl += 4) {
        if (tl >= pt) {
          tl -= pt;
          ++owner;
          peer = mapa_u32(recv0, (uint32_t)owner);
        }
        st_dsmem_f4(peer + (uint32_t)(((rank * pt + tl) * kDecBM + (e & 31) * 4) * 4),
                    reinterpret_cast<const float4*>(red)[t * (kDecBM / 4) + (e & 31)]);
      }
    }
  }
  __syncwarp();
  cluster_sync();  // every partial row is in its owner's receive buffer
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kDecBN);
  }
  if (warp < 2) return;

  // ------------------------------------------------------------ finisher (own shared memory only)
  dec_finish<FIN>(args, reinterpret_cast<const float4*>(recv), S, pt, ntok, tok0, row0, blk, warp, lane, kc, rpre);
}

// Launch with clusters of `cx` CTAs along x (and programmatic dependent launch when enabled).
template <typename... KArgs, typename... Args2>
cudaError_t launch_clusters(void (*kernel)(KArgs...), unsigned grid, unsigned cx, unsigned block, size_t smem,
                            cudaStream_t s, Args2... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cx;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  prefer_max_smem(reinterpret_cast<const void*>(kernel));
  launch_counter().fetch_add(1, std::memory_order_relaxed);
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// XB_DECODE_CLUSTER=0 in the environment keeps the older decode entry points
// on the split-K workspace path (partials in global memory + a finishing kernel).
bool decode_cluster_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("XB_DECODE_CLUSTER");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// Cluster size for a decode linear of `blocks` 128-row weight blocks and
// `kblocks` 64-wide K blocks: about two CTAs per SM, at most 8 (portable
// cluster size), every CTA with at least one K block.
// Largest split-K cluster the decode linears may use: the portable 8, or up
// to 16 with XB_DECODE_CLUSTER_MAX=16 in the environment (non-portable
// cluster size; used only where every cluster of the grid is resident at once).
int decode_cluster_max() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("XB_DECODE_CLUSTER_MAX");
    int x = e ? atoi(e) : 8;
    v = x < 1 ? 1 : (x > kDecMaxCluster ? kDecMaxCluster : x);
  }
  return v;
}

bool decode_deep_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("XB_DECODE_DEEP");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

void decode_split(int blocks, int kblocks, int max_s, int* splits, int* kps) {
  int sms = 148;
  sm_count(&sms);
  int s = (2 * sms) / blocks;
  if (s > max_s) s = max_s;
  if (s > kblocks) s = kblocks;
  if (s < 1) s = 1;
  for (;; --s) {
    *kps = (kblocks + s - 1) / s;
    *splits = (kblocks + *kps - 1) / *kps;
    // the receive buffer holds splits * ceil(64 / splits) token rows (<= 72)
    if (*splits * ((kDecBN + *splits - 1) / *splits) <= kDecRecvBytes / (kDecBM * 4) || s == 1) break;
  }
}

bool al8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; }
bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Shapes and pointers the decode kernel takes (false: the older entry points
// use the split-K workspace path instead).
bool decode_fits(const void* X, const void* W, int64_t M, int64_t N, int64_t K, int64_t ldx, int64_t ldw) {
  return M >= 1 && M <= kDecBN && N >= 1 && N % 4 == 0 && K >= 1 && ldx >= K && ldw >= K &&
         N <= (int64_t)kDecBM * 65535 && X && W && tma_ok(X, ldx, 2) && tma_ok(W, ldw, 2);
}

// A pending norm of X: the statistics of its rows (as the residual form of
// this kernel writes them) and the norm's parameters.
struct DecInput {
  const void* x;
  int64_t m, ldx;
  const float* stats;  // null: X is used as is
  const void* nw;
  const void* nb;
  float eps;
  int kind;
};

template <int FIN>
int launch_decode(const DecInput& in, const void* W, int64_t N, int64_t K, int64_t ldw, DecArgs args,
                  cudaStream_t s, const char* what, char* err, size_t errlen) {
  DecMaps maps;
  memset(&maps, 0, sizeof(maps));
  int rc = make_map(&maps.w, W, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, N, ldw, kDecBK, kDecBM, err, errlen);
  if (rc) return rc;
  rc = make_map(&maps.x, in.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, in.m, in.ldx, kDecBK, kDecBN, err, errlen);
  if (rc) return rc;
  const int blocks = (int)((N + kDecBM - 1) / kDecBM);
  args.m = (int)in.m;
  args.n = (int)N;
  args.k = (int)K;
  args.kblocks = (int)((K + kDecBK - 1) / kDecBK);
  args.xstats = reinterpret_cast<const float2*>(in.stats);
  args.xnw = static_cast<const __nv_bfloat16*>(in.nw);
  args.xnb = static_cast<const __nv_bfloat16*>(in.nb);
  args.xeps = in.eps;
  args.xkind = in.kind;
  int sms = 148;
  sm_count(&sms);
  const bool xn = in.stats != nullptr;
  void (*kernel)(DecMaps, DecArgs) = nullptr;
  int smem = 0;
  for (int max_s = decode_cluster_max();;) {
    decode_split(blocks, args.kblocks, max_s, &args.splits, &args.kps);
    // one CTA per SM with a deep ring when the grid is small, two with a short
    // one (XB_DECODE_DEEP=0 in the environment: always the short ring)
    const bool deep = blocks * args.splits <= sms && decode_deep_enabled();
    kernel = xn ? (deep ? decode_linear_kernel<FIN, 7, true> : decode_linear_kernel<FIN, 3, true>)
                : (deep ? decode_linear_kernel<FIN, 7, false> : decode_linear_kernel<FIN, 3, false>);
    smem = (deep ? 7 : 3) * kDecStage + kDecRecvBytes + 1024;
    cudaError_t e = once_per_device(reinterpret_cast<const void*>(kernel), kOnceSmem, [&](int*) {
      cudaError_t r = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      // clusters above the portable 8 only when asked for (XB_DECODE_CLUSTER_MAX)
      if (r == cudaSuccess && decode_cluster_max() > 8)
        r = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      return r;
    });
    if (e != cudaSuccess) {
      set_err(err, errlen, "%s: kernel setup: %s", what, cudaGetErrorString(e));
      return XB_ERR_CUDA;
    }
    if (args.splits <= 8) break;
    // a cluster above the portable size: keep it only if all `blocks` clusters
    // are resident at once (one wave), else fall back to the portable size
    int fits = 0;
    const int sp = args.splits;
    e = once_per_device(reinterpret_cast<const void*>(kernel), kOnceClusters + sp, [&](int* v) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)sp);
      cfg.blockDim = dim3(192);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = (unsigned)sp;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      cudaError_t r = cudaOccupancyMaxActiveClusters(v, kernel, &cfg);
      if (r != cudaSuccess) {  // not schedulable at this size: record zero resident clusters
        cudaGetLastError();
        *v = 0;
      }
      return cudaSuccess;
    }, &fits);
    if (e != cudaSuccess) {
      set_err(err, errlen, "%s: kernel setup: %s", what, cudaGetErrorString(e));
      return XB_ERR_CUDA;
    }
    if (fits >= blocks) break;
    max_s = 8;
  }
  cudaError_t e = launch_clusters(kernel, (unsigned)(blocks * args.splits), (unsigned)args.splits, 192, smem, s, maps,
                                  args);
  if (e != cudaSuccess) {
    set_err(err, errlen, "%s: %s", what, cudaGetErrorString(e));
    return XB_ERR_CUDA;
  }
  return check_launch(what, err, errlen);
}

// Validation shared by the xb_decode_* entry points: X (and its pending norm)
// and W.  Returns XB_OK or an error code with the message set.
int decode_check(const DecInput& in, const void* W, int64_t N, int64_t K, int64_t ldw, const char* what, char* err,
                 size_t errlen) {
  if (!in.x || !W) {
    set_err(err, errlen, "%s: null pointer", what);
    return XB_ERR_INVALID;
  }
  if (in.m < 1 || in.m > kDecBN || N < 1 || K < 1 || in.ldx < K || ldw < K) {
    set_err(err, errlen, "%s: needs 1 <= M <= %d tokens, N, K >= 1 and pitches >= K", what, kDecBN);
    return XB_ERR_INVALID;
  }
  if (N % 4 || N > (int64_t)kDecBM * 65535 || !tma_ok(in.x, in.ldx, 2) || !tma_ok(W, ldw, 2)) {
    set_err(err, errlen, "%s: N %% 4 == 0 and 16-byte aligned X / W rows needed", what);
    return XB_ERR_UNSUPPORTED;
  }
  if (in.stats) {
    if (in.kind != 0 && in.kind != 1) {
      set_err(err, errlen, "%s: x_norm_kind must be 0 (RMSNorm) or 1 (LayerNorm)", what);
      return XB_ERR_INVALID;
    }
    if (!in.nw || K % 8 || !al16(in.nw) || (in.nb && !al16(in.nb)) || !al8(in.stats)) {
      set_err(err, errlen, "%s: a pending norm needs K %% 8 == 0, 16-byte aligned norm vectors and statistics",
              what);
      return XB_ERR_UNSUPPORTED;
    }
  }
  return XB_OK;
}

}  // namespace gemm
}  // namespace xb

extern "C" int xb_linear_small_plan(int64_t M, int64_t N, int64_t K, int has_residual, int* splits,
                                    size_t* workspace_bytes, char* err, size_t errlen) {
  if (M < 0 || N <= 0 || K <= 0 || !splits || !workspace_bytes) {
    set_err(err, errlen, "xb_linear_small_plan: bad arguments");
    return XB_ERR_INVALID;
  }
  *splits = small_m_splits(N, K);
  *workspace_bytes = (*splits > 1 || has_residual) ? (size_t)(*splits) * (size_t)M * (size_t)N * sizeof(float) : 0;
  return XB_OK;
}

extern "C" int xb_linear_small_bf16(const void* X, const void* W, const void* bias, const void* residual, void* Y,
                                    int64_t M, int64_t N, int64_t K, int64_t ldx, int64_t ldw, int64_t ldr,
                                    int64_t ldy, int out_dtype, int splits, void* workspace, size_t workspace_bytes,
                                    void* stream, char* err, size_t errlen) {
  const char* what = "xb_linear_small_bf16";
  cudaStream_t s = (cudaStream_t)stream;
  if (out_dtype != XB_DT_F32 && out_dtype != XB_DT_BF16) {
    set_err(err, errlen, "%s: out_dtype must be f32 or bf16", what);
    return XB_ERR_UNSUPPORTED;
  }
  int rc = check_common(X, W, Y, M, N, K, ldx, ldw, ldy, true, what, err, errlen);
  if (rc) return rc < 0 ? rc : XB_OK;
  if (K == 0) {
    set_err(err, errlen, "%s: K must be positive", what);
    return XB_ERR_INVALID;
  }
  if (residual && ldr < N) {
    set_err(err, errlen, "%s: residual row pitch shorter than N", what);
    return XB_ERR_INVALID;
  }
  if (!tma_ok(X, ldx, 2) || !tma_ok(W, ldw, 2)) {
    set_err(err, errlen, "%s: X/W must be 16-byte aligned with row pitches a multiple of 16 bytes", what);
    return XB_ERR_UNSUPPORTED;
  }
  if (out_dtype == XB_DT_BF16 && decode_cluster_enabled() && decode_fits(X, W, M, N, K, ldx, ldw) && al8(Y) &&
      ldy % 4 == 0 && (!bias || al8(bias)) && (!residual || (al8(residual) && ldr % 4 == 0))) {
    DecArgs a;
    memset(&a, 0, sizeof(a));
    a.bias = static_cast<const __nv_bfloat16*>(bias);
    a.y = static_cast<__nv_bfloat16*>(Y);
    a.ldy = ldy;
    a.residual = static_cast<const __nv_bfloat16*>(residual);
    a.ldr = ldr;
    const DecInput in{X, M, ldx, nullptr, nullptr, nullptr, 0.0f, 0};
    if (residual) return launch_decode<kFinResidual>(in, W, N, K, ldw, a, s, what, err, errlen);
    return launch_decode<kFinStore>(in, W, N, K, ldw, a, s, what, err, errlen);
  }
  if (splits <= 0) splits = small_m_splits(N, K);
  const int kblocks = (int)((K + 63) / 64);
  if (splits > kblocks) splits = kblocks;
  const int kps = (kblocks + splits - 1) / splits;
  splits = (kblocks + kps - 1) / kps;
  // swap-AB: the weight is the 128-row MMA operand, the tokens the 64-wide one
  Operands op{{W, nullptr}, {X, nullptr}, ldw, ldx};
  if (splits == 1 && !residual) {
    if (out_dtype == XB_DT_F32)
      return launch<kBf16, true, kOutF32, 64, true>(op, Y, bias, N, M, K, ldy, s, what, err, errlen);
    return launch<kBf16, true, kOutBf16, 64, true>(op, Y, bias, N, M, K, ldy, s, what, err, errlen);
  }
  const size_t need = (size_t)splits * (size_t)M * (size_t)N * sizeof(float);
  if (!workspace || workspace_bytes < need) {
    set_err(err, errlen, "%s: workspace of %zu bytes given, %zu needed (%d K slices)", what, workspace_bytes, need,
            splits);
    return XB_ERR_INVALID;
  }
  float* part = static_cast<float*>(workspace);
  rc = launch<kBf16, true, kOutF32, 64, true>(op, part, nullptr, N, M, K, N, s, what, err, errlen, splits, M * N);
  if (rc) return rc;
  const int64_t total = M * N;
  const bool vec = N % 4 == 0 && M <= 65535 && (!bias || (reinterpret_cast<uintptr_t>(bias) & 7) == 0) &&
                   (!residual || ((reinterpret_cast<uintptr_t>(residual) & 7) == 0 && ldr % 4 == 0)) &&
                   (reinterpret_cast<uintptr_t>(Y) & 15) == 0 && ldy % 4 == 0;
  if (vec) {
    const dim3 g4((unsigned)((N / 4 + 255) / 256), (unsigned)M);
    const __nv_bfloat16* bp = static_cast<const __nv_bfloat16*>(bias);
    const __nv_bfloat16* rp = static_cast<const __nv_bfloat16*>(residual);
    if (out_dtype == XB_DT_BF16)
      launch_k(splitk_reduce4_kernel<true>, g4, 256, 0, s, (const float*)part, splits, (int)M, (int)N, bp, rp, ldr, Y,
               ldy);
    else
      launch_k(splitk_reduce4_kernel<false>, g4, 256, 0, s, (const float*)part, splits, (int)M, (int)N, bp, rp, ldr,
               Y, ldy);
    return check_launch(what, err, errlen);
  }
  int64_t grid = (total + 255) / 256;
  if (grid > 148 * 16) grid = 148 * 16;
  if (out_dtype == XB_DT_BF16)
    launch_k(splitk_reduce_kernel<true>, (unsigned)grid, 256, 0, s, part, splits, M, N,
                                                               static_cast<const __nv_bfloat16*>(bias),
                                                               static_cast<const __nv_bfloat16*>(residual), ldr, Y,
                                                               ldy);
  else
    launch_k(splitk_reduce_kernel<false>, (unsigned)grid, 256, 0, s, part, splits, M, N,
                                                                static_cast<const __nv_bfloat16*>(bias),
                                                                static_cast<const __nv_bfloat16*>(residual), ldr, Y,
                                                                ldy);
  return check_launch(what, err, errlen);
}

extern "C" int xb_linear_small_swiglu_bf16(const void* X, const void* W, void* Y, int64_t M, int64_t n_out, int64_t K,
                                           int64_t ldx, int64_t ldw, int64_t ldy, void* workspace,
                                           size_t workspace_bytes, void* stream, char* err, size_t errlen) {
  const char* what = "xb_linear_small_swiglu_bf16";
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t N = 2 * n_out;
  int rc = check_common(X, W, Y, M, N, K, ldx, ldw, ldy + n_out, true, what, err, errlen);
  if (rc) return rc < 0 ? rc : XB_OK;
  if (K == 0 || ldy < n_out) {
    set_err(err, errlen, "%s: bad K or output pitch", what);
    return XB_ERR_INVALID;
  }
  if (!tma_ok(X, ldx, 2) || !tma_ok(W, ldw, 2)) {
    set_err(err, errlen, "%s: X/W must be 16-byte aligned with row pitches a multiple of 16 bytes", what);
    return XB_ERR_UNSUPPORTED;
  }
  int splits = small_m_splits(N, K);
  const size_t need = (size_t)splits * (size_t)M * (size_t)N * sizeof(float);
  if (!workspace || workspace_bytes < need) {
    set_err(err, errlen, "%s: workspace of %zu bytes given, %zu needed", what, workspace_bytes, need);
    return XB_ERR_INVALID;
  }
  Operands op{{W, nullptr}, {X, nullptr}, ldw, ldx};
  float* part = static_cast<float*>(workspace);
  rc = launch<kBf16, true, kOutF32, 64, true>(op, part, nullptr, N, M, K, N, s, what, err, errlen, splits, M * N);
  if (rc) return rc;
  const int kblocks = (int)((K + 63) / 64);
  const int kps = (kblocks + splits - 1) / splits;
  splits = (kblocks + kps - 1) / kps;  // the count launch() used
  const int64_t total = M * n_out;
  if (n_out % 4 == 0 && M <= 65535 && (reinterpret_cast<uintptr_t>(Y) & 7) == 0 && ldy % 4 == 0) {
    const dim3 g4((unsigned)((n_out / 4 + 255) / 256), (unsigned)M);
    launch_k(splitk_swiglu4_kernel<false>, g4, 256, 0, s, (const float*)part, splits, (int)M, (int)n_out,
             static_cast<__nv_bfloat16*>(Y), ldy);
    return check_launch(what, err, errlen);
  }
  int64_t grid = (total + 255) / 256;
  if (grid > 148 * 16) grid = 148 * 16;
  launch_k(splitk_swiglu_kernel, (unsigned)grid, 256, 0, s, (const float*)part, splits, M, n_out,
           static_cast<__nv_bfloat16*>(Y), ldy);
  return check_launch(what, err, errlen);
}

// Shared front half of the fused decode entries: the split-K partials of
// X @ W^T (swap-AB small-M GEMM) into the workspace; returns the K slices used.
static int small_partials(const void* X, const void* W, int64_t M, int64_t N, int64_t K, int64_t ldx, int64_t ldw,
                          void* workspace, size_t workspace_bytes, cudaStream_t s, const char* what, int* splits_out,
                          char* err, size_t errlen) {
  if (M <= 0 || M > 65535 || N <= 0 || K <= 0 || ldx < K || ldw < K) {
    set_err(err, errlen, "%s: bad shape", what);
    return XB_ERR_INVALID;
  }
  if (!X || !W) {
    set_err(err, errlen, "%s: null pointer", what);
    return XB_ERR_INVALID;
  }
  if (!tma_ok(X, ldx, 2) || !tma_ok(W, ldw, 2)) {
    set_err(err, errlen, "%s: X/W must be 16-byte aligned with row pitches a multiple of 16 bytes", what);
    return XB_ERR_UNSUPPORTED;
  }
  int splits = small_m_splits(N, K);
  const size_t need = (size_t)splits * (size_t)M * (size_t)N * sizeof(float);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15) != 0) {
    set_err(err, errlen, "%s: 16-byte aligned workspace of %zu bytes needed (%zu given)", what, need,
            workspace_bytes);
    return XB_ERR_INVALID;
  }
  Operands op{{W, nullptr}, {X, nullptr}, ldw, ldx};
  int rc = launch<kBf16, true, kOutF32, 64, true>(op, workspace, nullptr, N, M, K, N, s, what, err, errlen, splits,
                                                  M * N);
  if (rc) return rc;
  const int kblocks = (int)((K + 63) / 64);
  const int kps = (kblocks + splits - 1) / splits;
  *splits_out = (kblocks + kps - 1) / kps;  // the count launch() used
  return XB_OK;
}

extern "C" int xb_linear_small_rope_kv_bf16(const void* X, const void* W, const void* bias, const float* cos_t,
                                            const float* sin_t, void* q_out, void* k_cache, void* v_cache,
                                            int64_t batch, int64_t n_head, int64_t n_kv_head, int64_t head_dim,
                                            int64_t max_seq, int64_t pos_offset, int64_t K, int64_t ldx, int64_t ldw,
                                            void* workspace, size_t workspace_bytes, void* stream, char* err,
                                            size_t errlen) {
  const char* what = "xb_linear_small_rope_kv_bf16";
  cudaStream_t s = (cudaStream_t)stream;
  if (n_head <= 0 || n_kv_head <= 0 || n_head % n_kv_head || head_dim <= 0 || head_dim % 2 || pos_offset < 0 ||
      pos_offset >= max_seq) {
    set_err(err, errlen, "%s: bad head layout or position", what);
    return XB_ERR_INVALID;
  }
  if (!q_out || !k_cache || !v_cache || (!cos_t) != (!sin_t)) {
    set_err(err, errlen, "%s: null pointer", what);
    return XB_ERR_INVALID;
  }
  const int64_t N = (n_head + 2 * n_kv_head) * head_dim;
  if (decode_cluster_enabled() && decode_fits(X, W, batch, N, K, ldx, ldw) && head_dim % 8 == 0 &&
      kDecBM % head_dim == 0 && al8(q_out) && al8(k_cache) && al8(v_cache) && (!bias || al8(bias)) &&
      (!cos_t || (al16(cos_t) && al16(sin_t)))) {
    DecArgs a;
    memset(&a, 0, sizeof(a));
    a.bias = static_cast<const __nv_bfloat16*>(bias);
    a.cos_t = cos_t;
    a.sin_t = sin_t;
    a.q_out = static_cast<__nv_bfloat16*>(q_out);
    a.k_cache = static_cast<__nv_bfloat16*>(k_cache);
    a.v_cache = static_cast<__nv_bfloat16*>(v_cache);
    a.H = (int)n_head;
    a.KVH = (int)n_kv_head;
    a.D = (int)head_dim;
    a.smax = (int)max_seq;
    a.pos = (int)pos_offset;
    const DecInput in{X, batch, ldx, nullptr, nullptr, nullptr, 0.0f, 0};
    return launch_decode<kFinRopeKv>(in, W, N, K, ldw, a, s, what, err, errlen);
  }
  int splits = 1;
  int rc = small_partials(X, W, batch, N, K, ldx, ldw, workspace, workspace_bytes, s, what, &splits, err, errlen);
  if (rc) return rc;
  const int64_t per_token = (n_head + 2 * n_kv_head) * (head_dim / 2);
  constexpr int kSplitY = 4;  // CTAs per token
  const int64_t per_cta = (per_token + kSplitY - 1) / kSplitY;
  const int threads = per_cta >= 1024 ? 1024 : (int)((per_cta + 31) / 32 * 32);
  launch_k(reduce_rope_kv_kernel, dim3((unsigned)batch, kSplitY), threads, 0, s, (const float*)workspace, splits, (int)batch, (int)N,
           static_cast<const __nv_bfloat16*>(bias), cos_t, sin_t, static_cast<__nv_bfloat16*>(q_out),
           static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), (int)n_head, (int)n_kv_head,
           (int)head_dim, (int)max_seq, (int)pos_offset);
  return check_launch(what, err, errlen);
}

extern "C" int xb_linear_small_residual_norm_bf16(const void* X, const void* W, const void* bias, const void* residual,
                                                  void* Y, void* Yn, const void* norm_w, const void* norm_b, float eps,
                                                  int norm_kind, int64_t M, int64_t N, int64_t K, int64_t ldx,
                                                  int64_t ldw, int64_t ldr, int64_t ldy, int64_t ldn, void* workspace,
                                                  size_t workspace_bytes, void* stream, char* err, size_t errlen) {
  const char* what = "xb_linear_small_residual_norm_bf16";
  cudaStream_t s = (cudaStream_t)stream;
  if (norm_kind != 0 && norm_kind != 1) {
    set_err(err, errlen, "%s: norm_kind must be 0 (RMSNorm) or 1 (LayerNorm)", what);
    return XB_ERR_INVALID;
  }
  if (N % 4 || N > 4096 || ldr < N || ldy < N || ldn < N || ldr % 4 || ldy % 4 || ldn % 4) {
    set_err(err, errlen, "%s: rows must be whole 4-element groups of at most 4096 (N = %lld)", what, (long long)N);
    return XB_ERR_UNSUPPORTED;
  }
  if (!residual || !Y || !Yn || !norm_w) {
    set_err(err, errlen, "%s: null pointer", what);
    return XB_ERR_INVALID;
  }
  const void* ptrs[6] = {bias, residual, Y, Yn, norm_w, norm_b};
  for (const void* p : ptrs)
    if (p && (reinterpret_cast<uintptr_t>(p) & 7)) {
      set_err(err, errlen, "%s: bf16 vectors must be 8-byte aligned", what);
      return XB_ERR_UNSUPPORTED;
    }
  typedef __nv_bfloat16 bf;
  if (decode_cluster_enabled() && decode_fits(X, W, M, N, K, ldx, ldw)) {
    // the residual linear in one launch, then the row norm of its output
    DecArgs a;
    memset(&a, 0, sizeof(a));
    a.bias = static_cast<const bf*>(bias);
    a.y = static_cast<bf*>(Y);
    a.ldy = ldy;
    a.residual = static_cast<const bf*>(residual);
    a.ldr = ldr;
    const DecInput in{X, M, ldx, nullptr, nullptr, nullptr, 0.0f, 0};
    int rc = launch_decode<kFinResidual>(in, W, N, K, ldw, a, s, what, err, errlen);
    if (rc) return rc;
    return norm_kind == 0 ? xb_rms_norm(Y, norm_w, Yn, M, N, ldy, ldn, eps, XB_DT_BF16, stream, err, errlen)
                          : xb_layernorm(Y, norm_w, norm_b, Yn, M, N, ldy, ldn, eps, XB_DT_BF16, stream, err, errlen);
  }
  int splits = 1;
  int rc = small_partials(X, W, M, N, K, ldx, ldw, workspace, workspace_bytes, s, what, &splits, err, errlen);
  if (rc) return rc;
  if (norm_kind == 0)
    launch_k(reduce_residual_norm_kernel<0>, (unsigned)M, 256, 0, s, (const float*)workspace, splits, (int)M, (int)N,
             static_cast<const bf*>(bias), static_cast<const bf*>(residual), ldr, static_cast<bf*>(Y), ldy,
             static_cast<bf*>(Yn), ldn, static_cast<const bf*>(norm_w), static_cast<const bf*>(norm_b), eps);
  else
    launch_k(reduce_residual_norm_kernel<1>, (unsigned)M, 256, 0, s, (const float*)workspace, splits, (int)M, (int)N,
             static_cast<const bf*>(bias), static_cast<const bf*>(residual), ldr, static_cast<bf*>(Y), ldy,
             static_cast<bf*>(Yn), ldn, static_cast<const bf*>(norm_w), static_cast<const bf*>(norm_b), eps);
  return check_launch(what, err, errlen);
}

extern "C" int xb_linear_rope_kv_bf16(const void* X, const void* W, const void* bias, const float* cos_t,
                                      const float* sin_t, int rope_dup, void* q_out, void* k_cache, void* v_cache,
                                      int64_t batch, int64_t seq, int64_t n_head, int64_t n_kv_head,
                                      int64_t head_dim, int64_t max_seq, int64_t pos_offset, int64_t K, int64_t ldx,
                                      int64_t ldw, void* stream, char* err, size_t errlen) {
  const char* what = "xb_linear_rope_kv_bf16";
  if (head_dim != 64 || n_head <= 0 || n_kv_head <= 0 || n_head % n_kv_head || batch < 0 || seq <= 0 ||
      pos_offset < 0 || pos_offset + seq > max_seq || max_seq > INT32_MAX) {
    set_err(err, errlen, "%s: bad head layout (head_dim 64) or positions", what);
    return XB_ERR_INVALID;
  }
  const int64_t M = batch * seq, N = (n_head + 2 * n_kv_head) * head_dim;
  if (M == 0) return XB_OK;
  if (!X || !W || !q_out || !k_cache || !v_cache || (!cos_t) != (!sin_t) || K <= 0 || ldx < K || ldw < K ||
      M > INT32_MAX) {
    set_err(err, errlen, "%s: null pointer or bad shape", what);
    return XB_ERR_INVALID;
  }
  const void* outs[5] = {q_out, k_cache, v_cache, cos_t, sin_t};
  for (const void* p : outs)
    if (reinterpret_cast<uintptr_t>(p) & 15) {
      set_err(err, errlen, "%s: q / K / V buffers and RoPE tables must be 16-byte aligned", what);
      return XB_ERR_UNSUPPORTED;
    }
  if (!tma_ok(X, ldx, 2) || !tma_ok(W, ldw, 2)) {
    set_err(err, errlen, "%s: X/W must be 16-byte aligned with row pitches a multiple of 16 bytes", what);
    return XB_ERR_UNSUPPORTED;
  }
  Args a;
  memset(&a, 0, sizeof(a));
  a.q_out = q_out;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.cos_t = cos_t;
  a.sin_t = sin_t;
  a.H = (int)n_head;
  a.KVH = (int)n_kv_head;
  a.S = (int)seq;
  a.smax = (int)max_seq;
  a.pos = (int)pos_offset;
  a.rope_dup = rope_dup ? 1 : 0;
  Operands op{{X, nullptr}, {W, nullptr}, ldx, ldw};
  cudaStream_t s = (cudaStream_t)stream;
  if (use_pairs(M))
    return epi8_enabled()
               ? launch<kBf16, true, kOutQkv, 0, false, false, true, 8>(op, nullptr, bias, M, N, K, N, s, what, err,
                                                                        errlen, 1, 0, nullptr, nullptr, 0, 0, &a)
               : launch<kBf16, true, kOutQkv, 0, false, false, true>(op, nullptr, bias, M, N, K, N, s, what, err,
                                                                     errlen, 1, 0, nullptr, nullptr, 0, 0, &a);
  return launch<kBf16, true, kOutQkv>(op, nullptr, bias, M, N, K, N, s, what, err, errlen, 1, 0, nullptr, nullptr, 0, 0,
                                      &a);
}

extern "C" int xb_linear_residual_bf16(const void* X, const void* W, const void* bias, const void* residual, void* Y,
                                       int64_t M, int64_t N, int64_t K, int64_t ldx, int64_t ldw, int64_t ldr,
                                       int64_t ldy, void* stream, char* err, size_t errlen) {
  const char* what = "xb_linear_residual_bf16";
  cudaStream_t s = (cudaStream_t)stream;
  int rc = check_common(X, W, Y, M, N, K, ldx, ldw, ldy, true, what, err, errlen);
  if (rc) return rc < 0 ? rc : XB_OK;
  if (!residual || ldr < N) {
    set_err(err, errlen, "%s: residual missing or its pitch shorter than N", what);
    return XB_ERR_INVALID;
  }
  if (K == 0 || !tma_ok(X, ldx, 2) || !tma_ok(W, ldw, 2)) {
    set_err(err, errlen, "%s: K must be positive and X/W 16-byte aligned with 16-byte row pitches", what);
    return XB_ERR_UNSUPPORTED;
  }
  Operands op{{X, nullptr}, {W, nullptr}, ldx, ldw};
  if (use_pairs(M))
    return epi8_enabled()
               ? launch<kBf16, true, kOutBf16, 0, false, false, true, 8>(op, Y, bias, M, N, K, ldy, s, what, err,
                                                                         errlen, 1, 0, nullptr, residual, ldr)
               : launch<kBf16, true, kOutBf16, 0, false, false, true>(op, Y, bias, M, N, K, ldy, s, what, err, errlen,
                                                                      1, 0, nullptr, residual, ldr);
  return launch<kBf16, true, kOutBf16>(op, Y, bias, M, N, K, ldy, s, what, err, errlen, 1, 0, nullptr, residual,
                                      ldr);
}

extern "C" int xb_linear_gelu_bf16(const void* X, const void* W, const void* bias, void* Y, int64_t M, int64_t N,
                                   int64_t K, int64_t ldx, int64_t ldw, int64_t ldy, void* workspace,
                                   size_t workspace_bytes, void* stream, char* err, size_t errlen) {
  const char* what = "xb_linear_gelu_bf16";
  cudaStream_t s = (cudaStream_t)stream;
  int rc = check_common(X, W, Y, M, N, K, ldx, ldw, ldy, true, what, err, errlen);
  if (rc) return rc < 0 ? rc : XB_OK;
  if (K == 0 || !tma_ok(X, ldx, 2) || !tma_ok(W, ldw, 2)) {
    set_err(err, errlen, "%s: K must be positive and X/W 16-byte aligned with 16-byte row pitches", what);
    return XB_ERR_UNSUPPORTED;
  }
  if (M > 64) {
    Operands op{{X, nullptr}, {W, nullptr}, ldx, ldw};
    if (use_pairs(M))
      return epi8_enabled()
                 ? launch<kBf16, true, kOutBf16, 0, false, false, true, 8>(op, Y, bias, M, N, K, ldy, s, what, err,
                                                                           errlen, 1, 0, nullptr, nullptr, 0, 1)
                 : launch<kBf16, true, kOutBf16, 0, false, false, true>(op, Y, bias, M, N, K, ldy, s, what, err,
                                                                        errlen, 1, 0, nullptr, nullptr, 0, 1);
    return launch<kBf16, true, kOutBf16>(op, Y, bias, M, N, K, ldy, s, what, err, errlen, 1, 0, nullptr, nullptr, 0,
                                        1);
  }
  // few tokens: split-K partials, then the reduction applies bias and GELU
  int splits = 1;
  if (N % 4 || (reinterpret_cast<uintptr_t>(Y) & 15) || ldy % 4 || (bias && (reinterpret_cast<uintptr_t>(bias) & 7))) {
    set_err(err, errlen, "%s: few-token form needs N %% 4 == 0 and aligned bias / output", what);
    return XB_ERR_UNSUPPORTED;
  }
  if (decode_cluster_enabled() && decode_fits(X, W, M, N, K, ldx, ldw) && (!bias || al8(bias))) {
    DecArgs a;
    memset(&a, 0, sizeof(a));
    a.bias = static_cast<const __nv_bfloat16*>(bias);
    a.y = static_cast<__nv_bfloat16*>(Y);
    a.ldy = ldy;
    a.act = 1;
    const DecInput in{X, M, ldx, nullptr, nullptr, nullptr, 0.0f, 0};
    return launch_decode<kFinStore>(in, W, N, K, ldw, a, s, what, err, errlen);
  }
  rc = small_partials(X, W, M, N, K, ldx, ldw, workspace, workspace_bytes, s, what, &splits, err, errlen);
  if (rc) return rc;
  const dim3 g4((unsigned)((N / 4 + 255) / 256), (unsigned)M);
  launch_k(splitk_reduce4_kernel<true, true>, g4, 256, 0, s, (const float*)workspace, splits, (int)M, (int)N,
           static_cast<const __nv_bfloat16*>(bias), (const __nv_bfloat16*)nullptr, (int64_t)0, Y, ldy);
  return check_launch(what, err, errlen);
}

extern "C" int xb_linear_swiglu_bf16(const void* X, const void* W, void* Y, int64_t M, int64_t n_out, int64_t K,
                                     int64_t ldx, int64_t ldw, int64_t ldy, void* workspace, size_t workspace_bytes,
                                     void* stream, char* err, size_t errlen) {
  const char* what = "xb_linear_swiglu_bf16";
  cudaStream_t s = (cudaStream_t)stream;
  if (n_out <= 0 || n_out % 64) {
    set_err(err, errlen, "%s: n_out must be a positive multiple of 64 (interleaved 64-row blocks)", what);
    return XB_ERR_UNSUPPORTED;
  }
  const int64_t N = 2 * n_out;
  int rc = check_common(X, W, Y, M, N, K, ldx, ldw, ldy + n_out, true, what, err, errlen);
  if (rc) return rc < 0 ? rc : XB_OK;
  if (K == 0 || ldy < n_out || !tma_ok(X, ldx, 2) || !tma_ok(W, ldw, 2)) {
    set_err(err, errlen, "%s: bad K / output pitch, or X/W not 16-byte aligned with 16-byte row pitches", what);
    return XB_ERR_UNSUPPORTED;
  }
  Operands op{{X, nullptr}, {W, nullptr}, ldx, ldw};
  if (M > 64) {
    if (use_pairs(M))
      return launch<kBf16, true, kOutSwiglu, 0, false, false, true>(op, Y, nullptr, M, N, K, ldy, s, what, err,
                                                                    errlen);
    return launch<kBf16, true, kOutSwiglu>(op, Y, nullptr, M, N, K, ldy, s, what, err, errlen);
  }
  // few tokens: one cluster split-K launch with the SwiGLU finisher
  if (decode_cluster_enabled() && decode_fits(X, W, M, N, K, ldx, ldw) && al8(Y) && ldy % 4 == 0) {
    DecArgs a;
    memset(&a, 0, sizeof(a));
    a.y = static_cast<__nv_bfloat16*>(Y);
    a.ldy = ldy;
    const DecInput in{X, M, ldx, nullptr, nullptr, nullptr, 0.0f, 0};
    return launch_decode<kFinSwiglu>(in, W, N, K, ldw, a, s, what, err, errlen);
  }
  // otherwise swap-AB split-K partials, then the interleaved SwiGLU finisher
  int splits = small_m_splits(N, K);
  const size_t need = (size_t)splits * (size_t)M * (size_t)N * sizeof(float);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15) ||
      (reinterpret_cast<uintptr_t>(Y) & 7) || ldy % 4) {
    set_err(err, errlen, "%s: 16-byte aligned workspace of %zu bytes and an 8-byte aligned output needed", what,
            need);
    return XB_ERR_INVALID;
  }
  Operands sop{{W, nullptr}, {X, nullptr}, ldw, ldx};
  rc = launch<kBf16, true, kOutF32, 64, true>(sop, workspace, nullptr, N, M, K, N, s, what, err, errlen, splits,
                                             M * N);
  if (rc) return rc;
  const int kblocks = (int)((K + 63) / 64);
  const int kps = (kblocks + splits - 1) / splits;
  splits = (kblocks + kps - 1) / kps;
  const dim3 g4((unsigned)((n_out / 4 + 255) / 256), (unsigned)M);
  launch_k(splitk_swiglu4_kernel<true>, g4, 256, 0, s, (const float*)workspace, splits, (int)M, (int)n_out,
           static_cast<__nv_bfloat16*>(Y), ldy);
  return check_launch(what, err, errlen);
}

// ---- decode-step linears with a pending input norm (one launch each) --------

#define XB_DECODE_INPUT                                                                         \
  const DecInput in{X, M, ldx, x_stats, x_norm_w, x_norm_b, x_eps, x_norm_kind};               \
  {                                                                                             \
    const int rc_ = decode_check(in, W, N, K, ldw, what, err, errlen);                          \
    if (rc_) return rc_;                                                                        \
  }

extern "C" int xb_decode_linear_bf16(const void* X, int64_t M, int64_t ldx, const float* x_stats,
                                     const void* x_norm_w, const void* x_norm_b, float x_eps, int x_norm_kind,
                                     const void* W, const void* bias, void* Y, int64_t N, int64_t K, int64_t ldw,
                                     int64_t ldy, int act, void* stream, char* err, size_t errlen) {
  const char* what = "xb_decode_linear_bf16";
  XB_DECODE_INPUT
  if (!Y || ldy < N || ldy % 4 || !al8(Y) || (bias && !al8(bias)) || (act != 0 && act != 1)) {
    set_err(err, errlen, "%s: bad output / bias (8-byte aligned, pitch %% 4 == 0) or act", what);
    return XB_ERR_INVALID;
  }
  DecArgs a;
  memset(&a, 0, sizeof(a));
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.y = static_cast<__nv_bfloat16*>(Y);
  a.ldy = ldy;
  a.act = act;
  return launch_decode<kFinStore>(in, W, N, K, ldw, a, (cudaStream_t)stream, what, err, errlen);
}

extern "C" int xb_decode_linear_rope_kv_bf16(const void* X, int64_t M, int64_t ldx, const float* x_stats,
                                             const void* x_norm_w, const void* x_norm_b, float x_eps,
                                             int x_norm_kind, const void* W, const void* bias, const float* cos_t,
                                             const float* sin_t, void* q_out, void* k_cache, void* v_cache,
                                             int64_t n_head, int64_t n_kv_head, int64_t head_dim, int64_t max_seq,
                                             int64_t pos_offset, int64_t K, int64_t ldw, void* stream, char* err,
                                             size_t errlen) {
  const char* what = "xb_decode_linear_rope_kv_bf16";
  if (n_head <= 0 || n_kv_head <= 0 || n_head % n_kv_head || head_dim <= 0 || head_dim % 8 ||
      kDecBM % head_dim || pos_offset < 0 || pos_offset >= max_seq) {
    set_err(err, errlen, "%s: bad head layout (head_dim %% 8 == 0 dividing 128) or position", what);
    return XB_ERR_INVALID;
  }
  const int64_t N = (n_head + 2 * n_kv_head) * head_dim;
  XB_DECODE_INPUT
  if (!q_out || !k_cache || !v_cache || (!cos_t) != (!sin_t) || !al8(q_out) || !al8(k_cache) || !al8(v_cache) ||
      (bias && !al8(bias)) || (cos_t && (!al16(cos_t) || !al16(sin_t)))) {
    set_err(err, errlen, "%s: null or unaligned output / bias (8-byte) or RoPE tables (16-byte)", what);
    return XB_ERR_INVALID;
  }
  DecArgs a;
  memset(&a, 0, sizeof(a));
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.cos_t = cos_t;
  a.sin_t = sin_t;
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  a.H = (int)n_head;
  a.KVH = (int)n_kv_head;
  a.D = (int)head_dim;
  a.smax = (int)max_seq;
  a.pos = (int)pos_offset;
  return launch_decode<kFinRopeKv>(in, W, N, K, ldw, a, (cudaStream_t)stream, what, err, errlen);
}

extern "C" int xb_decode_linear_swiglu_bf16(const void* X, int64_t M, int64_t ldx, const float* x_stats,
                                            const void* x_norm_w, const void* x_norm_b, float x_eps,
                                            int x_norm_kind, const void* W, void* Y, int64_t n_out, int64_t K,
                                            int64_t ldw, int64_t ldy, void* stream, char* err, size_t errlen) {
  const char* what = "xb_decode_linear_swiglu_bf16";
  if (n_out <= 0 || n_out % 64) {
    set_err(err, errlen, "%s: n_out must be a positive multiple of 64 (interleaved 64-row blocks)", what);
    return XB_ERR_UNSUPPORTED;
  }
  const int64_t N = 2 * n_out;
  XB_DECODE_INPUT
  if (!Y || ldy < n_out || ldy % 4 || !al8(Y)) {
    set_err(err, errlen, "%s: bad output (8-byte aligned, pitch %% 4 == 0)", what);
    return XB_ERR_INVALID;
  }
  DecArgs a;
  memset(&a, 0, sizeof(a));
  a.y = static_cast<__nv_bfloat16*>(Y);
  a.ldy = ldy;
  return launch_decode<kFinSwiglu>(in, W, N, K, ldw, a, (cudaStream_t)stream, what, err, errlen);
}

extern "C" int xb_decode_linear_residual_bf16(const void* X, int64_t M, int64_t ldx, const float* x_stats,
                                              const void* x_norm_w, const void* x_norm_b, float x_eps,
                                              int x_norm_kind, const void* W, const void* bias,
                                              const void* residual, void* Y, float* stats_out, int stats_kind,
                                              int64_t N, int64_t K, int64_t ldw, int64_t ldr, int64_t ldy,
                                              void* stream, char* err, size_t errlen) {
  const char* what = "xb_decode_linear_residual_bf16";
  XB_DECODE_INPUT
  if (!Y || !residual || ldy < N || ldr < N || ldy % 4 || ldr % 4 || !al8(Y) || !al8(residual) ||
      (bias && !al8(bias)) || (stats_out && (!al8(stats_out) || (stats_kind != 0 && stats_kind != 1)))) {
    set_err(err, errlen, "%s: bad output / residual / bias (8-byte aligned, pitches %% 4 == 0) or statistics", what);
    return XB_ERR_INVALID;
  }
  DecArgs a;
  memset(&a, 0, sizeof(a));
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.y = static_cast<__nv_bfloat16*>(Y);
  a.ldy = ldy;
  a.residual = static_cast<const __nv_bfloat16*>(residual);
  a.ldr = ldr;
  a.stats = reinterpret_cast<float2*>(stats_out);
  a.stats_kind = stats_kind;
  return launch_decode<kFinResidual>(in, W, N, K, ldw, a, (cudaStream_t)stream, what, err, errlen);
}
#undef XB_DECODE_INPUT

#include "decode_chain.cuh"

// ---- LM head + greedy next token --------------------------------------------

// idx[m] = argmax_n (X W^T)[m, n] per tile, then over the tiles.
namespace xb {
namespace gemm {
__global__ void __launch_bounds__(256) argmax_tiles_kernel(const uint2* __restrict__ cand, int tiles, int M,
                                                           int64_t cols, int64_t* __restrict__ idx) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sv[8];
  __shared__ int64_t si[8];
  const int m = blockIdx.x;
  float best = 0.0f;
  int64_t bi = cols;
  for (int t = threadIdx.x; t < tiles; t += 256) {
    const uint2 c = cand[(int64_t)t * M + m];
    if (argmax_better(best, bi, __uint_as_float(c.x), (int64_t)(int)c.y, cols)) {
      best = __uint_as_float(c.x);
      bi = (int)c.y;
    }
  }
#pragma unroll
  for (int o_ = 16; o_ > 0; o_ >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o_);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o_);
    if (argmax_better(best, bi, ov, oi, cols)) {
      best = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; ++w)
      if (argmax_better(best, bi, sv[w], si[w], cols)) {
        best = sv[w];
        bi = si[w];
      }
    idx[m] = bi;
  }
}
}  // namespace gemm
}  // namespace xb

extern "C" int xb_linear_argmax_workspace_size(int64_t M, int64_t N, size_t* bytes, char* err, size_t errlen) {
  if (!bytes || M < 0 || N < 0) {
    set_err(err, errlen, "xb_linear_argmax_workspace_size: bad arguments");
    return XB_ERR_INVALID;
  }
  *bytes = (size_t)((N + 127) / 128) * (size_t)M * 8u;
  return XB_OK;
}

extern "C" int xb_linear_argmax_bf16(const void* X, const void* W, int64_t M, int64_t N, int64_t K, int64_t ldx,
                                     int64_t ldw, int64_t* idx, void* workspace, size_t workspace_bytes,
                                     void* stream, char* err, size_t errlen) {
  const char* what = "xb_linear_argmax_bf16";
  cudaStream_t s = (cudaStream_t)stream;
  if (M <= 0 || M > 65535 || N <= 0 || N > ((int64_t)1 << 30) || K <= 0 || ldx < K || ldw < K || !X || !W || !idx) {
    set_err(err, errlen, "%s: bad shape or null pointer", what);
    return XB_ERR_INVALID;
  }
  if (!tma_ok(X, ldx, 2) || !tma_ok(W, ldw, 2)) {
    set_err(err, errlen, "%s: X/W must be 16-byte aligned with row pitches a multiple of 16 bytes", what);
    return XB_ERR_UNSUPPORTED;
  }
  const int tiles = (int)((N + 127) / 128);
  const size_t need = (size_t)tiles * (size_t)M * 8u;
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 7)) {
    set_err(err, errlen, "%s: 8-byte aligned workspace of %zu bytes needed (%zu given)", what, need, workspace_bytes);
    return XB_ERR_INVALID;
  }
  Operands op{{W, nullptr}, {X, nullptr}, ldw, ldx};  // swap-AB: vocabulary rows x tokens
  int rc = launch<kBf16, true, kOutArgmax, 64, true>(op, workspace, nullptr, N, M, K, M, s, what, err, errlen);
  if (rc) return rc;
  launch_k(argmax_tiles_kernel, dim3((unsigned)M), 256, 0, s, (const uint2*)workspace, tiles, (int)M, (int64_t)N, idx);
  return check_launch(what, err, errlen);
}

extern "C" int xb_matmul_sharded(const void* A, const void* B_shard, void* const* C_ranks, void* const* signal_ranks,
                                 int world, int rank, int64_t M, int64_t N_shard, int64_t K, int64_t lda, int64_t ldb,
                                 int64_t ldc, uint64_t epoch, uint64_t timeout_ns, int dtype, void* stream, char* err,
                                 size_t errlen) {
  const char* what = "xb_matmul_sharded";
  cudaStream_t s = (cudaStream_t)stream;
  if (world < 1 || world > 8 || rank < 0 || rank >= world || !C_ranks || !signal_ranks) {
    set_err(err, errlen, "%s: world must be 1..8 with a C and a signal pointer per rank", what);
    return XB_ERR_INVALID;
  }
  if (epoch == 0 || timeout_ns == 0) {
    set_err(err, errlen, "%s: epoch (1 for the first call on a signal buffer) and timeout_ns must be positive", what);
    return XB_ERR_INVALID;
  }
  if (ldc < (int64_t)world * N_shard) {
    set_err(err, errlen, "%s: ldc %lld shorter than world * N_shard", what, (long long)ldc);
    return XB_ERR_INVALID;
  }
  if (dtype != XB_DT_I8 && dtype != XB_DT_BF16) {
    set_err(err, errlen, "%s: dtype must be int8 or bf16", what);
    return XB_ERR_UNSUPPORTED;
  }
  if (M <= 0 || N_shard <= 0 || K <= 0) {
    set_err(err, errlen, "%s: M, N_shard and K must be positive", what);
    return XB_ERR_INVALID;
  }
  const int esz = dtype == XB_DT_I8 ? 1 : 2;
  const int osz = dtype == XB_DT_I8 ? 4 : 2;
  int rc = check_common(A, B_shard, C_ranks[rank], M, N_shard, K, lda, ldb, ldc, false, what, err, errlen);
  if (rc) return rc < 0 ? rc : XB_OK;
  if (!tma_ok(A, lda, esz) || !tma_ok(B_shard, ldb, esz)) {
    set_err(err, errlen, "%s: A/B must be 16-byte aligned with row pitches a multiple of 16 bytes", what);
    return XB_ERR_UNSUPPORTED;
  }
  PeerArgs pa;
  pa.world = world;
  pa.rank = rank;
  pa.epoch = epoch;
  pa.timeout_ns = timeout_ns;
  for (int r = 0; r < world; ++r) {
    if (!C_ranks[r] || !signal_ranks[r]) {
      set_err(err, errlen, "%s: null peer pointer for rank %d", what, r);
      return XB_ERR_INVALID;
    }
    // this rank's column block inside rank r's C
    pa.peers[r] = static_cast<char*>(C_ranks[r]) + (size_t)rank * N_shard * osz;
    pa.signals[r] = static_cast<uint64_t*>(signal_ranks[r]);
  }
  Operands op{{A, nullptr}, {B_shard, nullptr}, lda, ldb};
  void* local = pa.peers[rank];
  if (dtype == XB_DT_I8)
    return use_pairs(M) ? launch<kInt8, false, kOutI32, 0, false, true, true>(op, local, nullptr, M, N_shard, K, ldc,
                                                                              s, what, err, errlen, 1, 0, &pa)
                        : launch<kInt8, false, kOutI32, 0, false, true>(op, local, nullptr, M, N_shard, K, ldc, s,
                                                                        what, err, errlen, 1, 0, &pa);
  return use_pairs(M) ? launch<kBf16, false, kOutBf16, 0, false, true, true>(op, local, nullptr, M, N_shard, K, ldc, s,
                                                                             what, err, errlen, 1, 0, &pa)
                      : launch<kBf16, false, kOutBf16, 0, false, true>(op, local, nullptr, M, N_shard, K, ldc, s, what,
                                                                       err, errlen, 1, 0, &pa);
}

extern "C" int xb_device_status(void* stream, int* status, char* err, size_t errlen) {
  if (!status) {
    set_err(err, errlen, "xb_device_status: null output");
    return XB_ERR_INVALID;
  }
  cudaStream_t s = (cudaStream_t)stream;
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(status, g_gemm_status, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(g_gemm_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    set_err(err, errlen, "xb_device_status: %s", cudaGetErrorString(e));
    return XB_ERR_CUDA;
  }
  return XB_OK;
}

// ---- causal prefill attention on tcgen05 ----------------------------------------
//
// FlashAttention-style causal GQA attention (head_dim 64) for a prefill chunk,
// the numerics of examples/qwen2_5/kernels/attention.py:27-122: per key tile
// S = (Q K^T) * scale with the bounds and causal masks, m_new = max(m,
// rowmax S), alpha = exp(m - m_new), P = exp(S - m_new),
// acc = alpha * acc + bf16(P) @ V, l = alpha * l + rowsum(P), out = acc / l
// (exponentials in base 2 on the pre-scaled S).
//
// A unit is 128 query rows of one (sequence, head); key tiles of 64 keys.
// Two persistent CTAs per SM walk the units.  Warp 0 loads each unit's Q and
// its K / V tiles into a three-slot ring with TMA (3-D
// tensor maps whose key extent is the context length, so keys past it arrive
// as zeros).  Warp 1 issues the tcgen05 MMAs: S_j = Q K_j^T into one of two
// 64-column TMEM buffers, then, once P_j is in shared memory, P_j V_j into one
// of two more (a fresh accumulator per tile).  Warps 2-5 own one query row per
// thread: the row's scores come straight from TMEM (no cross-thread
// reductions), bf16(P) goes into one of two 128-byte-swizzled K-major tiles,
// and the tile's P V is folded into the row's fp32 accumulator in registers.
// Everything is double-buffered, so the MMAs of S_{j+1} and P_j V_j run while
// the softmax works on tile j and folds tile j - 1: the softmax warps stream
// through the tiles instead of waiting on each hand-off.  Two CTAs share an
// SM (97 KB shared memory, 256 TMEM columns each), and the units with the
// most key tiles come first.  Every wait is bounded (XB_ERR_TIMEOUT through
// the GEMM status word).
namespace xb {
namespace gemm {

constexpr int kAtBQ = 128;                 // query rows per CTA (TMEM lanes)
constexpr int kAtBK = 64;                  // keys per tile
constexpr int kAtQBytes = kAtBQ * 128;     // Q tile: 128 rows x 64 bf16
constexpr int kAtKVBytes = kAtBK * 128;    // K or V tile: 64 keys x 64 bf16
constexpr int kAtStages = 3;               // K / V ring slots
constexpr int kAtPBytes = kAtBQ * 128;     // P tile: 128 rows x 64 keys bf16
constexpr int kAtSmem = kAtQBytes + kAtStages * 2 * kAtKVBytes + 2 * kAtPBytes + 1024;

// two floats -> packed bf16 pair, the first in the low half (lower address)
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

struct alignas(64) AtMaps {
  CUtensorMap q;  // [B * H][S][64]
  CUtensorMap k;  // [B * KVH][total][64] (cache rows, extent = keys in context)
  CUtensorMap v;
};

struct AtArgs {
  __nv_bfloat16* out;  // [B * S][H * 64]
  int H, KVH, S, total, pos, nqt, nbh;
  float scale_log2;
};

// Unit u (query tile, sequence * head) of the causal prefill: the query tiles
// with the most key tiles come first.
struct AtUnit {
  int b, h, kvh, bh, qs, rows, nkt;
};
__device__ __forceinline__ AtUnit at_unit(const AtArgs& a, int u) {
  AtUnit t;
  const int qt = a.nqt - 1 - u / a.nbh;
  t.bh = u % a.nbh;
  t.b = t.bh / a.H;
  t.h = t.bh - t.b * a.H;
  t.kvh = t.h / (a.H / a.KVH);
  t.qs = qt * kAtBQ;
  t.rows = min(kAtBQ, a.S - t.qs);
  const int kmax = min(a.total, a.pos + t.qs + t.rows);  // keys the last row sees
  t.nkt = (kmax + kAtBK - 1) / kAtBK;
  return t;
}

// Persistent: each CTA walks units blockIdx.x, blockIdx.x + gridDim.x, ...;
// barrier phases, ring slots and TMEM buffers continue across units (tile
// counters are global to the CTA), so the next unit's Q and K / V loads and
// its first scores overlap the current unit's last tiles.
__global__ void __launch_bounds__(192, 2) attn_prefill_tc_kernel(const __grid_constant__ AtMaps maps,
                                                                  const AtArgs args) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full, q_empty, drain_bar;
  __shared__ __align__(8) uint64_t s_full[2], s_empty[2], p_full[2], o_full, o_empty;
  __shared__ __align__(8) uint64_t kv_full[kAtStages], kv_empty[kAtStages];
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base_u32 = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - smem_u32(smem_raw));
  const uint32_t sQ = base_u32, sKV = base_u32 + kAtQBytes, sP = sKV + kAtStages * 2 * kAtKVBytes;
  uint8_t* sPg = smem + kAtQBytes + kAtStages * 2 * kAtKVBytes;
  const int units = args.nqt * args.nbh;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&q_empty, 1);
    mbar_init(&drain_bar, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
      mbar_init(&p_full[i], 128);
    }
    mbar_init(&o_full, 1);    // one P V accumulated into O
    mbar_init(&o_empty, 128);  // a unit's O read by the softmax warps
    for (int i = 0; i < kAtStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&maps.q);
    prefetch_tmap(&maps.k);
    prefetch_tmap(&maps.v);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  // TMEM columns: S buffers [0, 64) and [64, 128), the output accumulator O [128, 192)
  pdl_wait();  // Q and the caches are written by the previous kernel
  pdl_trigger();

  auto fail = [&]() {
    atomicExch(&g_gemm_status, XB_ERR_TIMEOUT);
    abort_flag = 1;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t issued[kAtStages];
#pragma unroll
      for (int i = 0; i < kAtStages; ++i) issued[i] = 0;
      int g = 0, lu = 0;  // tiles and units of this CTA so far
      bool ok = true, q_issued = false;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++lu) {
        const AtUnit t = at_unit(args, u);
        // Q of this unit once the previous unit's last S MMA has read the old one
        if (lu > 0 && !mbar_wait(&q_empty, (lu - 1) & 1, kWaitLimit, &abort_flag)) {
          fail();
          break;
        }
        mbar_arrive_expect_tx(&q_full, kAtQBytes);
        tma_load_3d(smem, &maps.q, &q_full, 0, t.qs, t.bh);
        q_issued = true;
        const int kvrow = t.b * args.KVH + t.kvh;
        for (int j = 0; j < t.nkt; ++j, ++g) {
          const int st = g % kAtStages;
          if (!mbar_wait(&kv_empty[st], ((g / kAtStages) & 1) ^ 1, kWaitLimit, &abort_flag)) {
            fail();
            ok = false;
            break;
          }
          uint8_t* dst = smem + kAtQBytes + st * 2 * kAtKVBytes;
          mbar_arrive_expect_tx(&kv_full[st], 2 * kAtKVBytes);
          tma_load_3d(dst, &maps.k, &kv_full[st], 0, j * kAtBK, kvrow);
          tma_load_3d(dst + kAtKVBytes, &maps.v, &kv_full[st], 0, j * kAtBK, kvrow);
          issued[st] = g / kAtStages + 1;
        }
      }
      // every load issued must have landed before the CTA exits (also after an abort)
      uint64_t deadline = 0;
      if (q_issued && !mbar_wait_deadline(&q_full, (lu - 1) & 1, &deadline, kWaitLimit)) fail();
      for (int st = 0; st < kAtStages; ++st)
        if (issued[st] && !mbar_wait_deadline(&kv_full[st], (issued[st] - 1) & 1, &deadline, kWaitLimit)) fail();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdS = umma_idesc(1, 1, 1, 0, 0, kAtBQ, kAtBK);  // Q (K-major) x K tile (K-major)
      constexpr uint32_t kIdO = umma_idesc(1, 1, 1, 0, 1, kAtBQ, 64);     // P (K-major) x V tile (MN-major)
      bool any = false, ok = true;
      // P_g V_g accumulated into O once P_g is written (and O rescaled where
      // the softmax moved its base); the first tile of a unit starts O afresh,
      // after the softmax has read the previous unit's O
      auto pv = [&](int gi, bool first, int ulu) -> bool {
        const int pb_i = gi & 1;
        if (!mbar_wait(&p_full[pb_i], (gi >> 1) & 1, kWaitLimit, &abort_flag)) return false;
        if (first && ulu > 0 && !mbar_wait(&o_empty, (ulu - 1) & 1, kWaitLimit, &abort_flag)) return false;
        tc_fence_after();
        const uint32_t sv = sKV + (gi % kAtStages) * 2 * kAtKVBytes + kAtKVBytes;
        const uint32_t pb = sP + pb_i * kAtPBytes;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)  // keys in steps of 16
          mma_f16(tmem_base + 128, umma_desc_sw128(pb + ks * 32, 16, 1024),
                  umma_desc_sw128(sv + ks * 16 * 128, kAtKVBytes, 1024), kIdO, (!first || ks > 0) ? 1u : 0u);
        tc_commit(&o_full);
        tc_commit(&kv_empty[gi % kAtStages]);
        return true;
      };
      int g = 0, lu = 0;
      int pend_g = -1, pend_lu = 0;  // the tile whose P V is still to issue
      bool pend_first = false;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++lu) {
        const AtUnit t = at_unit(args, u);
        if (!mbar_wait(&q_full, lu & 1, kWaitLimit, &abort_flag)) {
          fail();
          break;
        }
        for (int j = 0; j < t.nkt; ++j, ++g) {
          // S_g into S buffer g & 1 (its previous scores, S_{g-2}, read by the softmax)
          const int st = g % kAtStages, sb = g & 1;
          if (!mbar_wait(&kv_full[st], (g / kAtStages) & 1, kWaitLimit, &abort_flag) ||
              (g >= 2 && !mbar_wait(&s_empty[sb], ((g - 2) >> 1) & 1, kWaitLimit, &abort_flag))) {
            fail();
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sk = sKV + st * 2 * kAtKVBytes;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)  // head dim in steps of 16
            mma_f16(tmem_base + sb * 64, umma_desc_sw128(sQ + ks * 32, 16, 1024),
                    umma_desc_sw128(sk + ks * 32, 16, 1024), kIdS, ks > 0 ? 1u : 0u);
          any = true;
          tc_commit(&s_full[sb]);
          if (j == t.nkt - 1) tc_commit(&q_empty);  // the unit's last S: Q may be replaced
          if (pend_g >= 0 && !pv(pend_g, pend_first, pend_lu)) {
            fail();
            ok = false;
            break;
          }
          pend_g = g;
          pend_first = j == 0;
          pend_lu = lu;
        }
      }
      if (ok && pend_g >= 0 && !pv(pend_g, pend_first, pend_lu)) fail();
      if (any) {  // every issued MMA completes before TMEM is released (also after an abort)
        tc_commit(&drain_bar);
        uint64_t deadline = 0;
        if (!mbar_wait_deadline(&drain_bar, 0, &deadline, kWaitLimit)) fail();
      }
    }
  } else {
    // ------------------------------------------------------------ softmax: one query row per thread
    // O accumulates in TMEM across the unit's key tiles.  P is taken relative
    // to a per-row base that moves only when the tile's max exceeds it by more
    // than 2^8 (P <= 256 otherwise, exact in bf16's range); a warp with such a
    // row rescales its rows of O in TMEM before the tile's P V is issued.
    const int q4 = warp & 3;  // TMEM lane quarter
    const int r = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    constexpr float kRebase = 8.0f;  // log2 of the largest P kept without rescaling
    bool ok = true;
    int g = 0;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const AtUnit t = at_unit(args, u);
      const int qpos = args.pos + t.qs + r;  // absolute position of this row
      float m = -INFINITY, l = 0.0f;  // m: the base of P (log2 units)
      for (int j = 0; j < t.nkt; ++j, ++g) {
        const int sb = g & 1;
        if (!mbar_wait(&s_full[sb], (g >> 1) & 1, kWaitLimit, &abort_flag)) {
          fail();
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sv[64];
        tmem_ld_32x32b_x32(tmem_base + sb * 64 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_ld_32x32b_x32(tmem_base + sb * 64 + 32 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(&s_empty[sb]);  // S buffer free for S_{g+2}
        const int k0 = j * kAtBK;
        const bool whole = k0 + kAtBK <= args.total && k0 + kAtBK - 1 <= qpos;  // no key of the tile masked
        // Raw scores (the scale is positive, so the max of the raw scores
        // scales to the max of the scaled ones); masked keys become -inf.  Row
        // max and row sum run as eight interleaved partial chains.
        float s[64];
        float mx8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = -INFINITY;
        if (whole) {
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            s[c] = __uint_as_float(sv[c]);
            mx8[c & 7] = fmaxf(mx8[c & 7], s[c]);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            const int key = k0 + c;
            s[c] = (key < args.total && key <= qpos) ? __uint_as_float(sv[c]) : -INFINITY;
            mx8[c & 7] = fmaxf(mx8[c & 7], s[c]);
          }
        }
        const float mxr = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        const float mn = fmaxf(m, mxr * args.scale_log2);
        // first tile: the base is the row max; later tiles: a warp moves the
        // bases of its rows only when one of them outgrew its base by 2^8
        const bool rebase = j == 0 || __any_sync(0xffffffffu, mn > m + kRebase);
        float alpha = 1.0f;
        if (rebase) {
          alpha = (j == 0 || m == -INFINITY) ? 0.0f : ex2_approx(m - mn);
          m = mn;
        }
        const float base = m == -INFINITY ? 0.0f : m;
        float rs8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) rs8[i] = 0.0f;
#pragma unroll
        for (int c = 0; c < 64; ++c) {  // P = exp2(S * scale - base): one FMA and one exponential
          s[c] = ex2_approx(fmaf(s[c], args.scale_log2, -base));
          rs8[c & 7] += s[c];
        }
        l = l * alpha + (((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7])));
        // bf16(P_g) row r -> P buffer g & 1 (read last by P_{g-2} V, complete:
        // waited in the previous tile); 16-byte chunk c8 at c8 ^ (r & 7) of the
        // 128-byte-swizzled K-major tile
        uint8_t* pt = sPg + sb * kAtPBytes + r * 128;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          uint4 w;
          w.x = pack_bf16x2(s[c8 * 8 + 0], s[c8 * 8 + 1]);
          w.y = pack_bf16x2(s[c8 * 8 + 2], s[c8 * 8 + 3]);
          w.z = pack_bf16x2(s[c8 * 8 + 4], s[c8 * 8 + 5]);
          w.w = pack_bf16x2(s[c8 * 8 + 6], s[c8 * 8 + 7]);
          *reinterpret_cast<uint4*>(pt + ((c8 ^ (r & 7)) << 4)) = w;
        }
        fence_proxy_async_smem();  // P, before the MMA (async proxy) reads it
        if (j > 0) {
          // P_{g-1} V is in O; rescale O's rows to the new bases before P_g V adds to it
          if (!mbar_wait(&o_full, (g - 1) & 1, kWaitLimit, &abort_flag)) {
            fail();
            ok = false;
            break;
          }
          tc_fence_after();
          if (rebase) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              uint32_t ov[32];
              tmem_ld_32x32b_x32(tmem_base + 128 + h * 32 + lane_off, ov);
              tmem_ld_wait();
#pragma unroll
              for (int c = 0; c < 32; ++c) ov[c] = __float_as_uint(__uint_as_float(ov[c]) * alpha);
              tmem_st_32x32b_x32(tmem_base + 128 + h * 32 + lane_off, ov);
            }
            tmem_st_wait();
          }
          tc_fence_before();
        }
        mbar_arrive(&p_full[sb]);
      }
      if (!ok) break;
      // the unit's last P V, then O: read, released for the next unit, normalised
      if (!mbar_wait(&o_full, (g - 1) & 1, kWaitLimit, &abort_flag)) {
        fail();
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t ov[64];
      tmem_ld_32x32b_x32(tmem_base + 128 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&ov[0]));
      tmem_ld_32x32b_x32(tmem_base + 128 + 32 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&ov[32]));
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&o_empty);
      if (r < t.rows) {
        const float inv = l > 0.0f ? 1.0f / l : 0.0f;
        __nv_bfloat16* op = args.out + ((int64_t)t.b * args.S + t.qs + r) * ((int64_t)args.H * 64) + t.h * 64;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(ov[c8 * 8 + 0]) * inv, __uint_as_float(ov[c8 * 8 + 1]) * inv);
          w.y = pack_bf16x2(__uint_as_float(ov[c8 * 8 + 2]) * inv, __uint_as_float(ov[c8 * 8 + 3]) * inv);
          w.z = pack_bf16x2(__uint_as_float(ov[c8 * 8 + 4]) * inv, __uint_as_float(ov[c8 * 8 + 5]) * inv);
          w.w = pack_bf16x2(__uint_as_float(ov[c8 * 8 + 6]) * inv, __uint_as_float(ov[c8 * 8 + 7]) * inv);
          *reinterpret_cast<uint4*>(op + c8 * 8) = w;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 256);
  }
}

// 3-D map [outer2][outer1][64 bf16] with 128-byte swizzle, box {64, box1, 1}.
int make_map_3d_sw128(CUtensorMap* map, const void* ptr, uint64_t outer1, uint64_t outer2, uint64_t ld1,
                      uint64_t ld2, uint32_t box1, char* err, size_t errlen) {
  EncodeTiledFn enc = encoder(err, errlen);
  if (!enc) return XB_ERR_CUDA;
  cuuint64_t dims[3] = {64, outer1, outer2};
  cuuint64_t strides[2] = {ld1 * 2, ld2 * 2};
  cuuint32_t box[3] = {64, box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_err(err, errlen, "cuTensorMapEncodeTiled failed (%d) for a [%llu][%llu][64] attention operand", (int)r,
            (unsigned long long)outer2, (unsigned long long)outer1);
    return XB_ERR_CUDA;
  }
  return XB_OK;
}

}  // namespace gemm

// Host side of the tcgen05 prefill attention (called by xb_attention_bf16 for
// seq > 1).  Returns XB_ERR_UNSUPPORTED when an operand breaks the TMA rules
// (the caller then uses the mma.sync kernel).
int attention_prefill_tc(const void* q, const void* k_cache, const void* v_cache, void* out, int64_t batch,
                         int64_t seq, int64_t n_head, int64_t n_kv_head, int64_t max_seq, int64_t pos_offset,
                         float scale_log2, cudaStream_t s, const char* what, char* err, size_t errlen) {
  using namespace gemm;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al16(q) || !al16(k_cache) || !al16(v_cache) || !al16(out)) return XB_ERR_UNSUPPORTED;
  const int64_t total = pos_offset + seq;
  const int64_t nqt = (seq + kAtBQ - 1) / kAtBQ;
  const int64_t nbh = batch * n_head;
  if (nqt * nbh > 0x7fffffffLL || total > 0x7fffffffLL) return XB_ERR_UNSUPPORTED;
  AtMaps maps;
  memset(&maps, 0, sizeof(maps));
  int rc = make_map_3d_sw128(&maps.q, q, (uint64_t)seq, (uint64_t)nbh, 64, (uint64_t)(seq * 64), kAtBQ, err, errlen);
  if (rc) return rc;
  rc = make_map_3d_sw128(&maps.k, k_cache, (uint64_t)total, (uint64_t)(batch * n_kv_head), 64,
                         (uint64_t)(max_seq * 64), kAtBK, err, errlen);
  if (rc) return rc;
  rc = make_map_3d_sw128(&maps.v, v_cache, (uint64_t)total, (uint64_t)(batch * n_kv_head), 64,
                         (uint64_t)(max_seq * 64), kAtBK, err, errlen);
  if (rc) return rc;
  AtArgs args;
  args.out = static_cast<__nv_bfloat16*>(out);
  args.H = (int)n_head;
  args.KVH = (int)n_kv_head;
  args.S = (int)seq;
  args.total = (int)total;
  args.pos = (int)pos_offset;
  args.nqt = (int)nqt;
  args.nbh = (int)nbh;
  args.scale_log2 = scale_log2;
  cudaError_t e = once_per_device(reinterpret_cast<const void*>(attn_prefill_tc_kernel), kOnceSmem, [](int*) {
    return cudaFuncSetAttribute(attn_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAtSmem);
  });
  if (e != cudaSuccess) {
    set_err(err, errlen, "%s: kernel setup: %s", what, cudaGetErrorString(e));
    return XB_ERR_CUDA;
  }
  int sms = 148;
  sm_count(&sms);
  const int64_t units = nqt * nbh;
  const int64_t grid = units < 2 * (int64_t)sms ? units : 2 * (int64_t)sms;  // two resident CTAs per SM
  launch_k(attn_prefill_tc_kernel, dim3((unsigned)grid), 192, kAtSmem, s, maps, args);
  return check_launch(what, err, errlen);
}

}  // namespace xb
