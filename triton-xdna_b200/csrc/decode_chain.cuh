// Decode chain: several decode-step linears in ONE persistent launch.
//
// A decode step of a decoder layer is a chain of small linears (64 tokens at
// most): o_proj + residual, gate/up + SwiGLU, down_proj + residual, and the
// next layer's QKV + RoPE + KV write.  Each is latency-bound on its own (a few
// MB of weights, 5-9 us of launch, set-up, split-K reduction and finisher).
// This kernel runs up to kChMaxPhases of them back to back inside one grid:
//
//   * clusters of kChS CTAs split K as the one-launch decode linear does
//     (partials reduced through distributed shared memory, the same fixed
//     rank order, the same finishers), but each cluster takes 128-row weight
//     blocks ("units") of every phase in turn: u = cluster, cluster + clusters,
//     ...
//   * phases are separated by a grid-wide barrier (a counter in global
//     memory, bounded spin): phase p + 1 reads what phase p wrote;
//   * weights do not depend on the barrier: the producer warp streams them
//     through the ring across phase boundaries, and every weight tile the
//     CTA will use is requested into L2 at the start, so the DRAM traffic of
//     the whole chain overlaps its latency-bound steps;
//   * X of a phase (this rank's K slice, all tokens) is loaded once per phase
//     and stays in shared memory for all of the cluster's units, normalised
//     in place when the phase has a pending norm;
//   * two TMEM accumulators and two receive buffers let the MMAs of a unit
//     and its partial-sum exchange overlap the finisher of the previous one.
//     The exchange is flow-controlled by cluster mbarriers (full / free)
//     instead of cluster-wide barriers, so the producer and MMA warps never
//     stop for the epilogue.
// Every wait is bounded; a CTA that gives up raises the launch's abort word,
// which every other wait of the grid also watches.

namespace xb {
namespace gemm {

constexpr int kChS = 8;                                  // CTAs per cluster (K split)
constexpr int kChStages = 3;                             // weight ring slots
constexpr int kChXMax = 10;                              // resident X tiles: K <= kChXMax * 64 * kChS
constexpr int kChMaxPhases = 4;
constexpr int kChWBytes = kDecBM * 128;                  // weight tile: 128 rows x 64 bf16
constexpr int kChXBytes = kDecBN * 128;                  // X tile: 64 tokens x 64 bf16
constexpr int kChRecvFloats = kDecBN * kDecBM;           // one receive buffer: [group token slot][row]
constexpr int kChRedBytes = kDecBN * kDecBM * 4;              // this CTA's partial [token][row]
constexpr int kChSmem =
    kChStages * kChWBytes + kChXMax * kChXBytes + 2 * kChRecvFloats * 4 + kChRedBytes + 1024;

// What a phase needs besides its tensor maps; copied into shared memory at
// the start of the launch (parameter reads at a run-time phase index go
// through the constant cache, whose first-touch misses cost ~0.5 us each on
// the finisher's critical path).
struct ChMeta {
  DecArgs a;   // finisher arguments (as the one-launch decode linear takes them)
  int fin;     // Fin
  int xnorm;   // X carries a pending norm (a.xstats ...)
  int units;   // 128-row weight blocks
  int split;   // CTAs of a cluster sharing a unit (8, 4, 2 or 1)
  int kps;     // K blocks per CTA of the group
  int nsplit;  // CTAs of the group that hold K blocks: ceil(kblocks / kps)
};
static_assert(sizeof(ChMeta) % 4 == 0, "copied as 32-bit words");

struct ChPhase {
  CUtensorMap w;  // W [N, K] K-major, 64 x 128 boxes
  CUtensorMap x;  // X [M, K] K-major, 64 x 64 boxes (rows past M read as zero)
  ChMeta m;
};

struct ChParams {
  ChPhase ph[kChMaxPhases];
  unsigned* sync;  // [0] grid arrivals, [1] CTAs done, [2] abort; all zero between launches
  int nph;
};
static_assert(sizeof(ChParams) <= 4000, "kernel parameters stay within the classic 4 KB");

__device__ __forceinline__ unsigned ld_acquire_gpu_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_volatile_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
// L2 prefetch of one tile of a tensor map (no shared memory, no completion)
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int32_t c0, int32_t c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1)
               : "memory");
}

// Arrivals (weight n) on an mbarrier of any CTA of the cluster.  The relaxed
// form is for signals that order only earlier reads: a release would also
// wait for this CTA's earlier global stores to be acknowledged.
__device__ __forceinline__ void mbar_arrive_cluster_n(uint32_t bar_cluster, uint32_t n) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(bar_cluster), "r"(n)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster_relaxed_n(uint32_t bar_cluster, uint32_t n) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(bar_cluster), "r"(n)
               : "memory");
}

// Bounded mbarrier wait that also gives up when this CTA (la) or any CTA of
// the grid (ga) has aborted.  CL: the phase is completed by arrivals from
// other CTAs of the cluster (acquire at cluster scope).
template <bool CL>
__device__ __forceinline__ bool ch_wait(uint64_t* bar, uint32_t parity, volatile int* la, const unsigned* ga) {
  auto probe = [&]() { return CL ? mbar_try_wait_cl(bar, parity) : mbar_try_wait(bar, parity); };
  if (probe()) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (probe()) return true;
    if ((i & 255) == 0) {
      if (*la || ld_volatile_u32(ga)) return false;
      if (globaltimer_ns() - t0 > kWaitLimit) return false;
    }
  }
}

// Runtime-dispatched finisher pieces (the phase kind is a kernel argument).
__device__ __forceinline__ DecConsts ch_consts(int fin, const DecArgs& a, int row0, int lane) {
  switch (fin) {
    case kFinStore: return dec_consts<kFinStore>(a, row0, lane);
    case kFinRopeKv: return dec_consts<kFinRopeKv>(a, row0, lane);
    case kFinSwiglu: return dec_consts<kFinSwiglu>(a, row0, lane);
    default: return dec_consts<kFinResidual>(a, row0, lane);
  }
}
__device__ __forceinline__ void ch_finish(int fin, const DecArgs& a, const float4* rv, int S, int pt, int ntok,
                                          int tok0, int row0, int blk, int warp, int lane, const DecConsts& kc,
                                          const float4 (&rpre)[kDecPre]) {
  switch (fin) {
    case kFinStore: dec_finish<kFinStore>(a, rv, S, pt, ntok, tok0, row0, blk, warp, lane, kc, rpre); break;
    case kFinRopeKv: dec_finish<kFinRopeKv>(a, rv, S, pt, ntok, tok0, row0, blk, warp, lane, kc, rpre); break;
    case kFinSwiglu: dec_finish<kFinSwiglu>(a, rv, S, pt, ntok, tok0, row0, blk, warp, lane, kc, rpre); break;
    default: dec_finish<kFinResidual>(a, rv, S, pt, ntok, tok0, row0, blk, warp, lane, kc, rpre); break;
  }
}

// One CTA: warp 0 streams weight tiles, warp 1 issues the MMAs, warps 2..5
// (the epilogue) load and normalise X, exchange partials and finish.  The
// epilogue never leaves its loops early: after an abort it runs on with every
// wait and every piece of work skipped, so its named barriers stay matched.
//
// K split per phase: s = split CTAs of a cluster share a unit (their K
// slices summed by the group's owners), so a cluster works on 8 / s units at
// once.  Every CTA of the grid runs the same number of unit slots in a phase
// (slots past the last unit exchange empty partials), which keeps the
// exchange barriers of all CTAs in step when the groups change between phases.
__global__ void __launch_bounds__(192, 1) decode_chain_kernel(const __grid_constant__ ChParams P) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t wfull[kChStages];
  __shared__ __align__(8) uint64_t wempty[kChStages];
  __shared__ __align__(8) uint64_t xfull;
  __shared__ __align__(8) uint64_t xready;
  __shared__ __align__(8) uint64_t tfull[2];
  __shared__ __align__(8) uint64_t tempty[2];
  __shared__ __align__(8) uint64_t rfull[2];
  __shared__ __align__(8) uint64_t rfree[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;
  __shared__ float s_mean[kDecBN], s_rstd[kDecBN];
  __shared__ ChMeta s_ph[kChMaxPhases];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t base_u32 = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - smem_u32(smem_raw));
  uint8_t* xs = smem + kChStages * kChWBytes;                         // resident X tiles
  float* recv = reinterpret_cast<float*>(xs + kChXMax * kChXBytes);  // [2][64 tokens of the group][128]
  float* red = recv + 2 * kChRecvFloats;                            // [64 tokens][128 rows]
  const uint32_t x_u32 = base_u32 + kChStages * kChWBytes;
  const int rank = (int)cluster_ctarank();
  const int cl = (int)blockIdx.x / kChS, ncl = (int)gridDim.x / kChS;
  unsigned* const sync = P.sync;
  const unsigned G = gridDim.x;
  const int nph = P.nph;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kChStages; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
    }
    mbar_init(&xfull, 1);
    mbar_init(&xready, 128);
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
      // arrivals are weighted by 8 / split, so these counts hold for every split:
      mbar_init(&rfull[a], kChS * 4);  // each source of the group, once per epilogue warp
      mbar_init(&rfree[a], kChS);      // each owner of the group, once its finisher is done
    }
    abort_flag = 0;
    mbar_fence_init();
  }
  {
    constexpr int kWords = (int)(sizeof(ChMeta) / 4);
    for (int i = threadIdx.x; i < nph * kWords; i += blockDim.x)
      reinterpret_cast<uint32_t*>(s_ph)[i] =
          reinterpret_cast<const uint32_t*>(&P.ph[i / kWords].m)[i % kWords];
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, 2 * kDecBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  cluster_sync();  // the peers' barriers exist before any remote arrival
  pdl_trigger();
  const uint32_t tmem_base = tmem_base_sh;
  auto fail = [&]() {
    atomicExch(&g_gemm_status, XB_ERR_TIMEOUT);
    abort_flag = 1;
    atomicExch(sync + 2, 1u);
  };
  // Geometry of a phase for this CTA: its group (split CTAs sharing a unit),
  // its K blocks [kb0, kb0 + nkb), its first unit and the unit stride, and
  // the number of unit slots every CTA runs.
  struct Geo {
    int s, r, g0, kb0, nkb, u0, ustep, slots;
  };
  auto geo = [&](const ChMeta& m) {
    Geo q;
    q.s = m.split;
    q.r = rank % q.s;  // rank within the group
    q.g0 = rank - q.r;  // the group's first rank
    q.kb0 = q.r * m.kps;
    q.nkb = max(0, min(q.kb0 + m.kps, m.a.kblocks) - q.kb0);
    const int ng = kChS / q.s;
    q.u0 = cl * ng + rank / q.s;
    q.ustep = ncl * ng;
    q.slots = (m.units + q.ustep - 1) / q.ustep;
    return q;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ weight producer
    if (lane == 0) {
      for (int p = 0; p < nph; ++p) {
        prefetch_tmap(&P.ph[p].w);
        prefetch_tmap(&P.ph[p].x);
      }
      // the ring's first fill, then every later tile of the launch into L2:
      // the chain's weight traffic runs at full DRAM rate under its
      // latency-bound steps (requested right after the first ring loads, so
      // those do not queue behind the prefetches)
      int it = 0;
      bool ok = true, prefetched = false;
      auto prefetch_rest = [&]() {
        int k = 0;
        for (int p = 0; p < nph; ++p) {
          const ChMeta& m = s_ph[p];
          const Geo q = geo(m);
          for (int u = q.u0; u < m.units; u += q.ustep)
            for (int i = 0; i < q.nkb; ++i, ++k)
              if (k >= kChStages) tma_prefetch_l2_2d(&P.ph[p].w, (q.kb0 + i) * kDecBK, u * kDecBM);
        }
        prefetched = true;
      };
      for (int p = 0; p < nph && ok; ++p) {
        const ChMeta& m = s_ph[p];
        const Geo q = geo(m);
        for (int u = q.u0; u < m.units && ok; u += q.ustep)
          for (int i = 0; i < q.nkb; ++i, ++it) {
            const int s = it % kChStages;
            if (it == kChStages && !prefetched) prefetch_rest();
            if (!ch_wait<false>(&wempty[s], ((it / kChStages) & 1) ^ 1, &abort_flag, sync + 2)) {
              fail();
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&wfull[s], kChWBytes);
            tma_load_2d(smem + s * kChWBytes, &P.ph[p].w, &wfull[s], (q.kb0 + i) * kDecBK, u * kDecBM);
          }
      }
      // the loads still in flight land before the CTA leaves (one time limit)
      uint64_t dl = 0;
      for (int j = it > kChStages ? it - kChStages : 0; j < it; ++j)
        if (!mbar_wait_deadline(&wfull[j % kChStages], (j / kChStages) & 1, &dl, kWaitLimit)) fail();
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc(1, 1, 1, 0, 0, kDecBM, kDecBN);
      int it = 0, ul = 0, xc = 0;
      bool ok = true, pending = false;
      for (int p = 0; p < nph && ok; ++p) {
        const ChMeta& m = s_ph[p];
        const Geo q = geo(m);
        if (q.u0 < m.units) {  // X is loaded only where the CTA has a unit
          if (!ch_wait<false>(&xready, xc & 1, &abort_flag, sync + 2)) {
            fail();
            break;
          }
          ++xc;
        }
        tc_fence_after();
        for (int j = 0; j < q.slots; ++j, ++ul) {
          const int a = ul & 1;
          const bool live = q.u0 + j * q.ustep < m.units;
          if (!ch_wait<false>(&tempty[a], ((ul >> 1) & 1) ^ 1, &abort_flag, sync + 2)) {
            fail();
            ok = false;
            break;
          }
          tc_fence_after();
          for (int i = 0; live && i < q.nkb; ++i, ++it) {
            const int s = it % kChStages;
            if (!ch_wait<false>(&wfull[s], (it / kChStages) & 1, &abort_flag, sync + 2)) {
              fail();
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t wa = base_u32 + s * kChWBytes, xa = x_u32 + i * kChXBytes;
#pragma unroll
            for (int ks = 0; ks < kDecBK / 16; ++ks)
              mma_f16(tmem_base + a * kDecBN, umma_desc_sw128(wa + ks * 32, 16, 1024),
                      umma_desc_sw128(xa + ks * 32, 16, 1024), idesc, (i > 0 || ks > 0) ? 1u : 0u);
            pending = true;
            tc_commit(&wempty[s]);
          }
          if (!ok) break;
          tc_commit(&tfull[a]);  // no MMAs (empty slot or K slice): completes at once
          pending = false;
        }
      }
      // the MMAs issued complete before the TMEM is released
      uint64_t dl = 0;
      if (pending) {
        tc_commit(&tfull[ul & 1]);
        if (!mbar_wait_deadline(&tfull[ul & 1], (ul >> 1) & 1, &dl, kWaitLimit)) fail();
      } else if (ul > 0) {
        if (!mbar_wait_deadline(&tfull[(ul - 1) & 1], ((ul - 1) >> 1) & 1, &dl, kWaitLimit)) fail();
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (128 threads)
    const int e = threadIdx.x - 64;  // 0 .. 127
    const int q4 = warp & 3;         // TMEM lane quarter this warp may read
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    int ul = 0, xf = 0, xissued = 0;
    for (int p = 0; p < nph; ++p) {
      const ChMeta& m = s_ph[p];
      const DecArgs& A = m.a;
      const Geo q = geo(m);
      const int pt = kDecBN / q.s;  // tokens each CTA of the group finishes
      const int tok0 = q.r * pt;
      const int ntok = max(0, min(A.m, tok0 + pt) - tok0);
      const unsigned weight = (unsigned)(kChS / q.s);  // exchange arrivals count 8 / split
      // ---- what phase p reads is complete: the previous kernel (phase 0) or
      // every CTA of this grid (the barrier counter reaches p * G)
      if (p == 0) {
        pdl_wait();
      } else {
        if (e == 0 && !abort_flag) {
          const unsigned target = (unsigned)p * G;
          uint64_t t0 = 0;
          for (uint32_t i = 0; ld_acquire_gpu_u32(sync) < target; ++i) {
            if ((i & 63) == 63) {
              if (ld_volatile_u32(sync + 2)) {
                abort_flag = 1;
                break;
              }
              const uint64_t now = globaltimer_ns();
              if (t0 == 0) {
                t0 = now;
              } else if (now - t0 > kWaitLimit) {
                fail();
                break;
              }
            }
          }
          fence_proxy_async_global();  // X is read through the async proxy next
        }
        epi_bar();
      }
      if (q.u0 < m.units) {
        // ---- this rank's K slice of X, all tokens, resident for the phase
        if (e == 0 && q.nkb > 0 && !abort_flag) {
          mbar_arrive_expect_tx(&xfull, q.nkb * kChXBytes);
          for (int i = 0; i < q.nkb; ++i)
            tma_load_2d(xs + i * kChXBytes, &P.ph[p].x, &xfull, (q.kb0 + i) * kDecBK, 0);
          ++xissued;
        }
        if (m.xnorm) {
          // per-token mean / rstd from the producer's block statistics, in block order
          if (e < kDecBN && !abort_flag) {
            const int t = e;
            float mean = 0.0f, rstd = 0.0f;
            if (t < A.m) {
              const int nb = (A.k + kDecBM - 1) / kDecBM;
              float na = 0.0f, ma = 0.0f, acc = 0.0f;
              for (int b0 = 0; b0 < nb; b0 += 8) {
                float2 st[8];
#pragma unroll
                for (int u = 0; u < 8; ++u)
                  st[u] = b0 + u < nb ? __ldcg(&A.xstats[(b0 + u) * kDecBN + t]) : make_float2(0.f, 0.f);
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                  if (b0 + u >= nb) break;
                  if (A.xkind == 0) {
                    acc += st[u].x;
                  } else {  // Chan et al.: merge (n_b, mean_b, M2_b) into the running (n, mean, M2)
                    const float nbk = (float)min(kDecBM, A.k - (b0 + u) * kDecBM);
                    const float n = na + nbk, delta = st[u].x - ma;
                    ma += delta * (nbk / n);
                    acc += st[u].y + delta * delta * (na * nbk / n);
                    na = n;
                  }
                }
              }
              mean = A.xkind == 0 ? 0.0f : ma;
              rstd = __frsqrt_rn(acc / (float)A.k + A.xeps);
            }
            s_mean[t] = mean;
            s_rstd[t] = rstd;
          }
          epi_bar();
        }
        if (q.nkb > 0) {
          if (e == 0 && !abort_flag && !ch_wait<false>(&xfull, xf & 1, &abort_flag, sync + 2)) fail();
          ++xf;
          epi_bar();
          if (m.xnorm && !abort_flag) {
            // thread e rewrites the 16-byte chunks (token (e >> 3) + 16 jj, K
            // elements 8 (e & 7) .. + 7) of every tile as bf16(norm(x))
            const int j = e & 7;
            for (int i = 0; i < q.nkb; ++i) {
              const int k0 = (q.kb0 + i) * kDecBK + j * 8;
              if (k0 >= A.k) continue;  // past K: zero-filled, stays zero
              const uint4 wraw = __ldg(reinterpret_cast<const uint4*>(A.xnw + k0));
              const uint4 braw = (A.xkind == 1 && A.xnb) ? __ldg(reinterpret_cast<const uint4*>(A.xnb + k0))
                                                         : make_uint4(0u, 0u, 0u, 0u);
              const __nv_bfloat162* wh = reinterpret_cast<const __nv_bfloat162*>(&wraw);
              const __nv_bfloat162* bh = reinterpret_cast<const __nv_bfloat162*>(&braw);
              uint8_t* xt = xs + i * kChXBytes;  // [64 tokens][128 bytes], 128-byte swizzle
#pragma unroll
              for (int jj = 0; jj < 4; ++jj) {
                const int r = (e >> 3) + 16 * jj;
                uint4* pp = reinterpret_cast<uint4*>(xt + r * 128 + ((j ^ (r & 7)) << 4));
                uint4 raw = *pp;
                __nv_bfloat162* hh = reinterpret_cast<__nv_bfloat162*>(&raw);
                const float mean = s_mean[r], rstd = s_rstd[r];
                if (A.xkind == 0) {
#pragma unroll
                  for (int q2 = 0; q2 < 4; ++q2)
                    hh[q2] = __floats2bfloat162_rn(
                        __fmul_rn(__fmul_rn(__low2float(hh[q2]), rstd), __low2float(wh[q2])),
                        __fmul_rn(__fmul_rn(__high2float(hh[q2]), rstd), __high2float(wh[q2])));
                } else {
#pragma unroll
                  for (int q2 = 0; q2 < 4; ++q2)
                    hh[q2] = __floats2bfloat162_rn(
                        (__low2float(hh[q2]) - mean) * rstd * __low2float(wh[q2]) + __low2float(bh[q2]),
                        (__high2float(hh[q2]) - mean) * rstd * __high2float(wh[q2]) + __high2float(bh[q2]));
                }
                *pp = raw;
              }
            }
          }
          fence_proxy_async_smem();  // these writes, before the MMAs' (async-proxy) reads
        }
        mbar_arrive(&xready);
      }
      // ---- the unit slots of this phase, software-pipelined: slot j's
      // partial is pushed before slot j - 1 is finished, so the wait for the
      // slowest group member's push overlaps this CTA's own push.  Slot ul
      // (counted over the launch) uses accumulator and receive buffer ul & 1.
      int pj = -1, pa = 0, pul = 0, pu = 0;
      bool plive = false;
      DecConsts pkc = {};
      float4 prpre[kDecPre];
      auto finish_pending = [&]() {
        if (e == 0 && !abort_flag && !ch_wait<true>(&rfull[pa], (pul >> 1) & 1, &abort_flag, sync + 2)) fail();
        epi_bar();
        if (plive && !abort_flag)
          ch_finish(m.fin, A, reinterpret_cast<const float4*>(recv + pa * kChRecvFloats), m.nsplit, pt, ntok, tok0,
                    pu * kDecBM, pu, warp, lane, pkc, prpre);
        // every epilogue thread has read receive buffer pa (the named barrier
        // orders those reads); the sources are told so without waiting for the
        // finisher's global stores
        epi_bar();
        if (e < q.s) mbar_arrive_cluster_relaxed_n(mapa_u32(smem_u32(&rfree[pa]), (uint32_t)(q.g0 + e)), weight);
      };
      for (int j = 0; j < q.slots; ++j, ++ul) {
        const int a = ul & 1;
        const int u = q.u0 + j * q.ustep;
        const bool live = u < m.units;
        DecConsts kc = {};
        float4 rpre[kDecPre];
#pragma unroll
        for (int v4 = 0; v4 < kDecPre; ++v4) rpre[v4] = z4;
        if (live) {
          kc = ch_consts(m.fin, A, u * kDecBM, lane);
          if (m.fin == kFinResidual) dec_rpre<kFinResidual>(A, ntok, tok0, u * kDecBM, warp, lane, rpre);
        }
        // receive buffers a of the group are free (slot ul - 2 finished) and
        // this CTA's accumulator a is final (one thread polls each barrier;
        // the named barrier passes the result on)
        if (e == 0 && !abort_flag) {
          if (!ch_wait<true>(&rfree[a], ((ul >> 1) & 1) ^ 1, &abort_flag, sync + 2) ||
              !ch_wait<false>(&tfull[a], (ul >> 1) & 1, &abort_flag, sync + 2))
            fail();
        }
        epi_bar();
        tc_fence_after();
        const bool push = live && q.nkb > 0 && !abort_flag;
        if (push) {
          // accumulator -> red [token][row] (thread = row), the TMEM
          // accumulator is then free for the next slot's MMAs
          const int row = q4 * 32 + lane;
#pragma unroll
          for (int h = 0; h < kDecBN / 32; ++h) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q4 * 32) << 16) + a * kDecBN + h * 32, v);
            tmem_ld_wait();
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) red[(h * 32 + jj) * kDecBM + row] = __uint_as_float(v[jj]);
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[a]);
        epi_bar();
        if (push) {
          // token t's row of the partial -> slot (q.r, t % pt) of its owner's
          // receive buffer: thread e sends rows (e & 31) * 4 .. + 3 of tokens
          // e / 32 + 4 k, one 16-byte store each (a warp: one 512-byte row).
          // Staged through shared memory: stores of register values straight
          // after the TMEM load ran ~0.5 us each (measured).
          const uint32_t recv_a = smem_u32(recv + a * kChRecvFloats);
          const float4* red4 = reinterpret_cast<const float4*>(red);
#pragma unroll 4
          for (int t = e >> 5; t < kDecBN; t += 4)
            st_dsmem_f4(mapa_u32(recv_a + (uint32_t)(((q.r * pt + t % pt) * kDecBM + (e & 31) * 4) * 4),
                                 (uint32_t)(q.g0 + t / pt)),
                        red4[t * (kDecBM / 4) + (e & 31)]);
        }
        // this warp's pushes, released to every owner of the group (lane o
        // arrives at owner o)
        __syncwarp();
        if (lane < q.s) mbar_arrive_cluster_n(mapa_u32(smem_u32(&rfull[a]), (uint32_t)(q.g0 + lane)), weight);
        if (pj >= 0) finish_pending();
        pj = j;
        pa = a;
        pul = ul;
        pu = u;
        plive = live;
        pkc = kc;
#pragma unroll
        for (int v4 = 0; v4 < kDecPre; ++v4) prpre[v4] = rpre[v4];
      }
      if (pj >= 0) finish_pending();
      // ---- this CTA's part of phase p is written: one arrival on the grid counter
      if (p + 1 < nph) {
        epi_bar();
        if (e == 0) {
          __threadfence();
          fence_proxy_async_global();
          red_release_gpu_add(sync, 1u);
        }
      }
    }
    // an X load still in flight lands before the CTA leaves
    if (e == 0 && xissued > 0) {
      uint64_t dl = 0;
      if (!mbar_wait_deadline(&xfull, (xissued - 1) & 1, &dl, kWaitLimit)) fail();
    }
    __syncwarp();
  }
  // no peer touches this CTA's shared memory after the cluster barrier
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * kDecBN);
  }
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(sync + 1, 1u) == G - 1) {  // the last CTA out: counters back to zero for the next launch
      atomicExch(sync, 0u);
      atomicExch(sync + 2, 0u);
      __threadfence();
      atomicExch(sync + 1, 0u);
    }
  }
}

// One xb_decode_phase -> kernel phase, with the checks of the matching
// single-launch entry point.
int chain_phase(const xb_decode_phase& d, ChPhase& ph, const char* what, char* err, size_t errlen) {
  if (d.kind < XB_DECODE_STORE || d.kind > XB_DECODE_RESIDUAL) {
    set_err(err, errlen, "%s: phase kind must be XB_DECODE_STORE .. XB_DECODE_RESIDUAL", what);
    return XB_ERR_INVALID;
  }
  const DecInput in{d.x, d.m, d.ldx, d.x_stats, d.x_norm_w, d.x_norm_b, d.x_eps, d.x_norm_kind};
  const int64_t N = d.n, K = d.k;
  int rc = decode_check(in, d.w, N, K, d.ldw, what, err, errlen);
  if (rc) return rc;
  DecArgs& a = ph.m.a;
  memset(&a, 0, sizeof(a));
  switch (d.kind) {
    case XB_DECODE_STORE:
      if (!d.y || d.ldy < N || d.ldy % 4 || !al8(d.y) || (d.bias && !al8(d.bias)) || (d.act != 0 && d.act != 1)) {
        set_err(err, errlen, "%s: bad output / bias (8-byte aligned, pitch %% 4 == 0) or act", what);
        return XB_ERR_INVALID;
      }
      a.act = d.act;
      break;
    case XB_DECODE_ROPE_KV:
      if (d.n_head <= 0 || d.n_kv_head <= 0 || d.n_head % d.n_kv_head || d.head_dim <= 0 || d.head_dim % 8 ||
          kDecBM % d.head_dim || d.pos_offset < 0 || d.pos_offset >= d.max_seq ||
          N != (d.n_head + 2 * d.n_kv_head) * d.head_dim) {
        set_err(err, errlen, "%s: bad head layout (n = (H + 2 KVH) * D, D %% 8 == 0 dividing 128) or position",
                what);
        return XB_ERR_INVALID;
      }
      if (!d.q_out || !d.k_cache || !d.v_cache || (!d.cos_t) != (!d.sin_t) || !al8(d.q_out) || !al8(d.k_cache) ||
          !al8(d.v_cache) || (d.bias && !al8(d.bias)) || (d.cos_t && (!al16(d.cos_t) || !al16(d.sin_t)))) {
        set_err(err, errlen, "%s: null or unaligned output / bias (8-byte) or RoPE tables (16-byte)", what);
        return XB_ERR_INVALID;
      }
      a.cos_t = d.cos_t;
      a.sin_t = d.sin_t;
      a.q_out = static_cast<__nv_bfloat16*>(d.q_out);
      a.k_cache = static_cast<__nv_bfloat16*>(d.k_cache);
      a.v_cache = static_cast<__nv_bfloat16*>(d.v_cache);
      a.H = (int)d.n_head;
      a.KVH = (int)d.n_kv_head;
      a.D = (int)d.head_dim;
      a.smax = (int)d.max_seq;
      a.pos = (int)d.pos_offset;
      break;
    case XB_DECODE_SWIGLU:
      if (N % 128 || !d.y || d.ldy < N / 2 || d.ldy % 4 || !al8(d.y) || d.bias) {
        set_err(err, errlen, "%s: SwiGLU needs n = 2 n_out with n_out %% 64 == 0, no bias and an 8-byte aligned "
                "output (pitch %% 4 == 0)", what);
        return XB_ERR_INVALID;
      }
      break;
    default:
      if (!d.y || !d.residual || d.ldy < N || d.ldr < N || d.ldy % 4 || d.ldr % 4 || !al8(d.y) ||
          !al8(d.residual) || (d.bias && !al8(d.bias)) ||
          (d.stats_out && (!al8(d.stats_out) || (d.stats_kind != 0 && d.stats_kind != 1)))) {
        set_err(err, errlen, "%s: bad output / residual / bias (8-byte aligned, pitches %% 4 == 0) or statistics",
                what);
        return XB_ERR_INVALID;
      }
      a.residual = static_cast<const __nv_bfloat16*>(d.residual);
      a.ldr = d.ldr;
      a.stats = reinterpret_cast<float2*>(d.stats_out);
      a.stats_kind = d.stats_kind;
      break;
  }
  if (d.kind != XB_DECODE_ROPE_KV) {
    a.y = static_cast<__nv_bfloat16*>(d.y);
    a.ldy = d.ldy;
  }
  if (d.kind != XB_DECODE_SWIGLU) a.bias = static_cast<const __nv_bfloat16*>(d.bias);
  a.m = (int)d.m;
  a.n = (int)N;
  a.k = (int)K;
  a.kblocks = (int)((K + kDecBK - 1) / kDecBK);
  a.xstats = reinterpret_cast<const float2*>(d.x_stats);
  a.xnw = static_cast<const __nv_bfloat16*>(d.x_norm_w);
  a.xnb = static_cast<const __nv_bfloat16*>(d.x_norm_b);
  a.xeps = d.x_eps;
  a.xkind = d.x_norm_kind;
  if ((a.kblocks + kChS - 1) / kChS > kChXMax) {
    set_err(err, errlen, "%s: K = %lld exceeds the chain's %d resident K blocks per CTA (K <= %d)", what,
            (long long)K, kChXMax, kChXMax * kDecBK * kChS);
    return XB_ERR_UNSUPPORTED;
  }
  ph.m.fin = d.kind;  // XB_DECODE_* match the Fin values
  ph.m.xnorm = d.x_stats != nullptr;
  ph.m.units = (int)((N + kDecBM - 1) / kDecBM);
  return XB_OK;
}

// The phase's tensor maps (after every phase of the chain passed its checks).
int chain_maps(const xb_decode_phase& d, ChPhase& ph, char* err, size_t errlen) {
  const int rc = make_map(&ph.w, d.w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d.k, d.n, d.ldw, kDecBK, kDecBM, err,
                          errlen);
  if (rc) return rc;
  return make_map(&ph.x, d.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d.k, d.m, d.ldx, kDecBK, kDecBN, err, errlen);
}
static_assert(kFinStore == XB_DECODE_STORE && kFinRopeKv == XB_DECODE_ROPE_KV && kFinSwiglu == XB_DECODE_SWIGLU &&
                  kFinResidual == XB_DECODE_RESIDUAL,
              "phase kinds are the finisher kinds");

}  // namespace gemm
}  // namespace xb

extern "C" int xb_decode_chain_bf16(const xb_decode_phase* phases, int n_phases, void* sync, void* stream,
                                    char* err, size_t errlen) {
  using namespace xb;
  using namespace xb::gemm;
  const char* what = "xb_decode_chain_bf16";
  if (!phases || n_phases < 1 || n_phases > kChMaxPhases || !sync || (reinterpret_cast<uintptr_t>(sync) & 3)) {
    set_err(err, errlen, "%s: needs 1..%d phases and a 4-byte aligned sync buffer", what, kChMaxPhases);
    return XB_ERR_INVALID;
  }
  ChParams P;
  memset(&P, 0, sizeof(P));
  for (int i = 0; i < n_phases; ++i) {
    const int rc = chain_phase(phases[i], P.ph[i], what, err, errlen);
    if (rc) return rc;
  }
  for (int i = 0; i < n_phases; ++i) {
    const int rc = chain_maps(phases[i], P.ph[i], err, errlen);
    if (rc) return rc;
  }
  P.nph = n_phases;
  P.sync = static_cast<unsigned*>(sync);
  void (*kernel)(ChParams) = decode_chain_kernel;
  cudaError_t e = once_per_device(reinterpret_cast<const void*>(kernel), kOnceSmem, [&](int*) {
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kChSmem);
  });
  // clusters resident at once: the grid barrier needs every CTA of the grid running
  int fits = 0;
  if (e == cudaSuccess)
    e = once_per_device(reinterpret_cast<const void*>(kernel), kOnceClusters + kChS, [&](int* v) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)kChS);
      cfg.blockDim = dim3(192);
      cfg.dynamicSmemBytes = kChSmem;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = (unsigned)kChS;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(v, kernel, &cfg) != cudaSuccess) {
        cudaGetLastError();
        *v = 0;
      }
      return cudaSuccess;
    }, &fits);
  if (e != cudaSuccess) {
    set_err(err, errlen, "%s: kernel setup: %s", what, cudaGetErrorString(e));
    return XB_ERR_CUDA;
  }
  if (fits < 1) {
    set_err(err, errlen, "%s: no %d-CTA cluster of the chain kernel fits on this device", what, kChS);
    return XB_ERR_UNSUPPORTED;
  }
  // every resident cluster takes part; each phase then splits K as little as
  // keeps all of them busy: halve the split while the units times the halved
  // split still cover the grid and the slices still fit the resident X tiles
  const int ncl = fits;
  for (int i = 0; i < n_phases; ++i) {
    ChMeta& m = P.ph[i].m;
    int sp = kChS;
    while (sp > 1 && (m.a.kblocks + sp / 2 - 1) / (sp / 2) <= kChXMax && m.units * (sp / 2) >= ncl * kChS) sp /= 2;
    m.split = sp;
    m.kps = (m.a.kblocks + sp - 1) / sp;
    m.nsplit = (m.a.kblocks + m.kps - 1) / m.kps;
    m.a.kps = m.kps;
    m.a.splits = m.nsplit;
  }
  e = launch_clusters(kernel, (unsigned)(ncl * kChS), (unsigned)kChS, 192, kChSmem, (cudaStream_t)stream, P);
  if (e != cudaSuccess) {
    set_err(err, errlen, "%s: %s", what, cudaGetErrorString(e));
    return XB_ERR_CUDA;
  }
  return check_launch(what, err, errlen);
}
