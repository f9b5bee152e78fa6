// Kernels of the Qwen2.5 decoder forward that are not plain GEMMs or norms:
// token embedding gather, rotary embedding fused with the KV-cache write,
// causal GQA attention for prefill and for single-token decode, and the
// greedy argmax over the vocabulary.
//
// Reference: examples/qwen2_5/model.py:824-901 (`_attention`: fused QKV
// projection, RoPE, KV-cache write, GQA, fused attention), 903-911
// (embedding), 1134-1179 (`generate`, greedy argmax);
// examples/qwen2_5/kernels/rope.py:20-67 (rotate-half RoPE in fp32);
// examples/qwen2_5/kernels/attention.py:27-122 (`fused_attention_kernel`:
// online softmax in fp32, P cast to bf16 before P@V, bf16 output).
//
// Layouts (all bf16 unless noted):
//   qkv      [M = B*S, (H + 2*KVH) * D]   output of the fused QKV linear
//   q        [B, H, S, D]                 roped queries
//   k/v cache[B, KVH, Smax, D]            per layer (model.py:1110-1132)
//   attn out [B, S, H*D]                  input of o_proj
//   cos/sin  [max_pos, D] fp32            tables of rope.py:20-35
#include "common.cuh"
#include "tc.cuh"

namespace xb {
namespace llm {

typedef __nv_bfloat16 bf16;

// ----------------------------------------------------------------------------- embedding

// out[m, :] = table[ids[m], :]; one warp per row, 16-byte vectors.
__global__ void __launch_bounds__(256) embedding_kernel(const bf16* __restrict__ table, const int64_t* __restrict__ ids,
                                                        bf16* __restrict__ out, int64_t rows, int64_t dim,
                                                        int64_t vocab, int* __restrict__ bad) {
  pdl_wait();
  pdl_trigger();
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  int64_t id = ids[row];
  if (id < 0 || id >= vocab) {  // out-of-range token: flag it, write zeros
    if (lane == 0) atomicExch(bad, 1);
    for (int64_t c = lane; c < dim; c += 32) out[row * dim + c] = __float2bfloat16_rn(0.0f);
    return;
  }
  const int4* src = reinterpret_cast<const int4*>(table + id * dim);
  int4* dst = reinterpret_cast<int4*>(out + row * dim);
  for (int64_t v = lane; v < dim / 8; v += 32) dst[v] = __ldg(src + v);
}

// out[m, :] = bf16(table[ids[m], :] + pos_table[pos_offset + m % seq, :]):
// token plus learned position embedding, one rounding of the fp32 sum (the
// bf16 + bf16 add of examples/gpt2/model.py:872-876).
__global__ void __launch_bounds__(256) embedding_pos_kernel(const bf16* __restrict__ table,
                                                            const bf16* __restrict__ pos_table,
                                                            const int64_t* __restrict__ ids, bf16* __restrict__ out,
                                                            int64_t rows, int64_t dim, int64_t vocab, int seq,
                                                            int pos_offset, int* __restrict__ bad) {
  pdl_wait();
  pdl_trigger();
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t id = ids[row];
  int4* dst = reinterpret_cast<int4*>(out + row * dim);
  if (id < 0 || id >= vocab) {  // out-of-range token: flag it, write zeros
    if (lane == 0) atomicExch(bad, 1);
    for (int64_t v = lane; v < dim / 8; v += 32) dst[v] = make_int4(0, 0, 0, 0);
    return;
  }
  const int4* a = reinterpret_cast<const int4*>(table + id * dim);
  const int4* p = reinterpret_cast<const int4*>(pos_table + (int64_t)(pos_offset + (int)(row % seq)) * dim);
  for (int64_t v = lane; v < dim / 8; v += 32) {
    int4 x = __ldg(a + v), y = __ldg(p + v);
    const bf16* xe = reinterpret_cast<const bf16*>(&x);
    const bf16* ye = reinterpret_cast<const bf16*>(&y);
    int4 o;
    bf16* oe = reinterpret_cast<bf16*>(&o);
#pragma unroll
    for (int e = 0; e < 8; ++e) oe[e] = __float2bfloat16_rn(__bfloat162float(xe[e]) + __bfloat162float(ye[e]));
    dst[v] = o;
  }
}

// ----------------------------------------------------------------------------- RoPE + KV write

// One CTA per token; thread j of the CTA handles head slot j / (D/2) and pair
// i = j % (D/2).  Head slots [0, H) are queries, [H, H+KVH) keys,
// [H+KVH, H+2KVH) values (copied unrotated).
// x_out[i] = x[i]*cos - x[i+D/2]*sin, x_out[i+D/2] = x[i+D/2]*cos + x[i]*sin,
// each product and sum rounded separately in fp32 as rope.py:63-66 does.
__global__ void __launch_bounds__(1024) rope_kv_kernel(const bf16* __restrict__ qkv, const float* __restrict__ cos_t,
                                                       const float* __restrict__ sin_t, bf16* __restrict__ q_out,
                                                       bf16* __restrict__ k_cache, bf16* __restrict__ v_cache, int S,
                                                       int H, int KVH, int D, int smax, int pos_offset) {
  pdl_wait();
  pdl_trigger();
  const int half = D / 2;
  const int slots = H + 2 * KVH;
  const int64_t m = blockIdx.x;  // token row b*S + s
  const int s = (int)(m % S);
  const int b = (int)(m / S);
  const int pos = pos_offset + s;
  const bf16* xrow = qkv + m * (int64_t)(slots * D);
  const bool rotate = cos_t != nullptr;  // no tables: heads are copied (learned positions)
  const float* cr = rotate ? cos_t + (int64_t)pos * D : nullptr;
  const float* sr = rotate ? sin_t + (int64_t)pos * D : nullptr;
  for (int j = threadIdx.x; j < slots * half; j += blockDim.x) {
    const int slot = j / half;
    const int i = j - slot * half;
    const bf16* x = xrow + slot * D;
    if (slot >= H + KVH) {  // value head: copy
      bf16* dst = v_cache + (((int64_t)b * KVH + (slot - H - KVH)) * smax + pos) * D;
      dst[i] = x[i];
      dst[i + half] = x[i + half];
      continue;
    }
    bf16* dst = slot < H ? q_out + (((int64_t)b * H + slot) * S + s) * D
                         : k_cache + (((int64_t)b * KVH + (slot - H)) * smax + pos) * D;
    if (!rotate) {
      dst[i] = x[i];
      dst[i + half] = x[i + half];
      continue;
    }
    const float x0 = __bfloat162float(x[i]);
    const float x1 = __bfloat162float(x[i + half]);
    const float y0 = __fadd_rn(__fmul_rn(x0, cr[i]), __fmul_rn(-x1, sr[i]));
    const float y1 = __fadd_rn(__fmul_rn(x1, cr[i + half]), __fmul_rn(x0, sr[i + half]));
    dst[i] = __float2bfloat16_rn(y0);
    dst[i + half] = __float2bfloat16_rn(y1);
  }
}

// The same RoPE + KV write for many tokens: a grid-stride loop over (token,
// head slot, pair of adjacent dims) items, 4-byte bf16x2 and 8-byte float2
// accesses, several tokens per CTA (one CTA per token left the block
// scheduler as the bottleneck of a 32768-token prefill).  Identical
// arithmetic: products and sums rounded separately in fp32.
__global__ void __launch_bounds__(256) rope_kv_flat_kernel(const bf16* __restrict__ qkv, const float* __restrict__ cos_t,
                                                           const float* __restrict__ sin_t, bf16* __restrict__ q_out,
                                                           bf16* __restrict__ k_cache, bf16* __restrict__ v_cache,
                                                           int64_t tokens, int S, int H, int KVH, int D, int smax,
                                                           int pos_offset) {
  pdl_wait();
  pdl_trigger();
  const int half = D / 2, hp = half / 2;  // pairs of dims per head slot
  const int slots = H + 2 * KVH;
  const int64_t per_tok = (int64_t)slots * hp;
  const int64_t total = tokens * per_tok;
  for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < total; it += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = it / per_tok;
    const int rem = (int)(it - m * per_tok);
    const int slot = rem / hp;
    const int i = (rem - slot * hp) * 2;
    const int s = (int)(m % S);
    const int b = (int)(m / S);
    const int pos = pos_offset + s;
    const bf16* x = qkv + m * (int64_t)(slots * D) + slot * D;
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(x + i);
    const __nv_bfloat162 c = *reinterpret_cast<const __nv_bfloat162*>(x + i + half);
    if (slot >= H + KVH) {
      bf16* dst = v_cache + (((int64_t)b * KVH + (slot - H - KVH)) * smax + pos) * D;
      *reinterpret_cast<__nv_bfloat162*>(dst + i) = a;
      *reinterpret_cast<__nv_bfloat162*>(dst + i + half) = c;
      continue;
    }
    bf16* dst = slot < H ? q_out + (((int64_t)b * H + slot) * S + s) * D
                         : k_cache + (((int64_t)b * KVH + (slot - H)) * smax + pos) * D;
    if (!cos_t) {
      *reinterpret_cast<__nv_bfloat162*>(dst + i) = a;
      *reinterpret_cast<__nv_bfloat162*>(dst + i + half) = c;
      continue;
    }
    const float2 c0 = *reinterpret_cast<const float2*>(cos_t + (int64_t)pos * D + i);
    const float2 c1 = *reinterpret_cast<const float2*>(cos_t + (int64_t)pos * D + i + half);
    const float2 s0 = *reinterpret_cast<const float2*>(sin_t + (int64_t)pos * D + i);
    const float2 s1 = *reinterpret_cast<const float2*>(sin_t + (int64_t)pos * D + i + half);
    const float x0a = __low2float(a), x0b = __high2float(a), x1a = __low2float(c), x1b = __high2float(c);
    const float y0a = __fadd_rn(__fmul_rn(x0a, c0.x), __fmul_rn(-x1a, s0.x));
    const float y0b = __fadd_rn(__fmul_rn(x0b, c0.y), __fmul_rn(-x1b, s0.y));
    const float y1a = __fadd_rn(__fmul_rn(x1a, c1.x), __fmul_rn(x0a, s1.x));
    const float y1b = __fadd_rn(__fmul_rn(x1b, c1.y), __fmul_rn(x0b, s1.y));
    *reinterpret_cast<__nv_bfloat162*>(dst + i) = __floats2bfloat162_rn(y0a, y0b);
    *reinterpret_cast<__nv_bfloat162*>(dst + i + half) = __floats2bfloat162_rn(y1a, y1b);
  }
}

// ----------------------------------------------------------------------------- prefill attention

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* smem_row) {
  const uint32_t addr = (uint32_t)__cvta_generic_to_shared(smem_row);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

constexpr int kHD = 64;        // head dim supported (Qwen2.5-0.5B)
constexpr int kBQ = 64;        // query rows per CTA (16 per warp)
constexpr int kBK = 64;        // keys per tile
constexpr int kPad = kHD + 8;  // smem row pitch (elements): conflict-free fragment loads

// Causal GQA attention on mma.sync (the fallback of the tcgen05 kernel in
// csrc/gemm.cu), FlashAttention-style: a CTA of 4 warps owns 64 query
// rows of one (batch, head); K/V tiles of 64 keys go through shared memory;
// S = Q K^T and O += P V run on mma.sync m16n8k16 (bf16 in, fp32 accumulate);
// the softmax is online in fp32 with exp2.  Query row s (absolute position
// pos_offset + s) sees keys 0 .. pos_offset + s, as attention.py:85-87.
__global__ void __launch_bounds__(128) attn_prefill_kernel(const bf16* __restrict__ q, const bf16* __restrict__ kc,
                                                           const bf16* __restrict__ vc, bf16* __restrict__ out, int H,
                                                           int KVH, int S, int smax, int pos_offset,
                                                           float scale_log2) {
  pdl_wait();
  pdl_trigger();
  __shared__ __align__(16) bf16 sK[2][kBK][kPad];  // double-buffered key / value tiles
  __shared__ __align__(16) bf16 sV[2][kBK][kPad];
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int kvh = h / (H / KVH);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int qw = blockIdx.x * kBQ + warp * 16;  // first query row of this warp
  const bf16* qp = q + ((int64_t)(b * H + h) * S) * kHD;
  const bf16* kp = kc + ((int64_t)(b * KVH + kvh) * smax) * kHD;
  const bf16* vp = vc + ((int64_t)(b * KVH + kvh) * smax) * kHD;

  uint32_t qa[4][4];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const int r0 = qw + g, r1 = qw + g + 8, c = kk * 16 + 2 * t;
    qa[kk][0] = r0 < S ? *reinterpret_cast<const uint32_t*>(qp + (int64_t)r0 * kHD + c) : 0u;
    qa[kk][1] = r1 < S ? *reinterpret_cast<const uint32_t*>(qp + (int64_t)r1 * kHD + c) : 0u;
    qa[kk][2] = r0 < S ? *reinterpret_cast<const uint32_t*>(qp + (int64_t)r0 * kHD + c + 8) : 0u;
    qa[kk][3] = r1 < S ? *reinterpret_cast<const uint32_t*>(qp + (int64_t)r1 * kHD + c + 8) : 0u;
  }

  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;

  const int total = pos_offset + S;  // keys in the cache after this chunk
  const int last_q = min(S, (int)blockIdx.x * kBQ + kBQ) - 1;
  const int kmax = min(total, pos_offset + last_q + 1);
  const int qa0 = pos_offset + qw + g, qa1 = qa0 + 8;  // absolute positions of this thread's rows

  // Tiles stream through two buffers with cp.async: tile i + 2 is requested
  // as soon as tile i has been consumed, so the copies overlap the math
  // (rows past the context are zero-filled, nothing read).
  const int ntiles = (kmax + kBK - 1) / kBK;
  auto issue = [&](int tile, int buf) {
    const int t0 = tile * kBK;
    for (int v = threadIdx.x; v < kBK * kHD / 8; v += 128) {
      const int row = v / (kHD / 8), c8 = (v % (kHD / 8)) * 8;
      const bool ok = t0 + row < total;
      const int64_t src = (int64_t)(ok ? t0 + row : 0) * kHD + c8;
      const uint32_t bytes = ok ? 16u : 0u;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                       (uint32_t)__cvta_generic_to_shared(&sK[buf][row][c8])),
                   "l"(kp + src), "r"(bytes)
                   : "memory");
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                       (uint32_t)__cvta_generic_to_shared(&sV[buf][row][c8])),
                   "l"(vp + src), "r"(bytes)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if (ntiles > 0) issue(0, 0);
  if (ntiles > 1) issue(1, 1);
  for (int it = 0; it < ntiles; ++it) {
    const int buf = it & 1, k0 = it * kBK;
    if (it + 1 < ntiles) asm volatile("cp.async.wait_group 1;" ::: "memory");
    else asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // every thread's copies of tile `it` have landed

    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&sK[buf][nt * 8 + g][kk * 16 + 2 * t]);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&sK[buf][nt * 8 + g][kk * 16 + 8 + 2 * t]);
        mma_bf16_16816(s[nt], qa[kk], b0, b1);
      }
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
    // a tile wholly inside the context and at or below the warp's first
    // query row needs no mask (every tile but the diagonal ones)
    const bool unmasked = k0 + kBK <= total && k0 + kBK - 1 <= pos_offset + qw;
    if (unmasked) {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        s[nt][0] *= scale_log2;
        s[nt][1] *= scale_log2;
        s[nt][2] *= scale_log2;
        s[nt][3] *= scale_log2;
        mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
        mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
      }
    } else {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = k0 + nt * 8 + 2 * t + (e & 1);
          const int qpos = e < 2 ? qa0 : qa1;
          const bool ok = key < total && key <= qpos;
          s[nt][e] = ok ? s[nt][e] * scale_log2 : -INFINITY;
          if (e < 2) mx0 = fmaxf(mx0, s[nt][e]);
          else mx1 = fmaxf(mx1, s[nt][e]);
        }
    }
#pragma unroll
    for (int o_ = 1; o_ <= 2; o_ <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o_));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o_));
    }
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float base0 = mn0 == -INFINITY ? 0.0f : mn0, base1 = mn1 == -INFINITY ? 0.0f : mn1;
    const float al0 = ex2_approx(m0 - base0), al1 = ex2_approx(m1 - base1);
    m0 = mn0;
    m1 = mn1;
    float rs0 = 0.0f, rs1 = 0.0f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = ex2_approx(s[nt][0] - base0);
      s[nt][1] = ex2_approx(s[nt][1] - base0);
      s[nt][2] = ex2_approx(s[nt][2] - base1);
      s[nt][3] = ex2_approx(s[nt][3] - base1);
      rs0 += s[nt][0] + s[nt][1];
      rs1 += s[nt][2] + s[nt][3];
    }
    l0 = l0 * al0 + rs0;
    l1 = l1 * al1 + rs1;
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) {
      o[dt][0] *= al0;
      o[dt][1] *= al0;
      o[dt][2] *= al1;
      o[dt][3] *= al1;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // keys kk*16 .. kk*16+15 of the tile
      uint32_t pa[4];
      pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dt = 0; dt < 8; dt += 2) {
        const int mi = lane >> 3, r = lane & 7;
        uint32_t vb[4];
        ldmatrix_x4_trans(vb, &sV[buf][kk * 16 + (mi & 1) * 8 + r][dt * 8 + (mi >> 1) * 8]);
        mma_bf16_16816(o[dt], pa, vb[0], vb[1]);
        mma_bf16_16816(o[dt + 1], pa, vb[2], vb[3]);
      }
    }
    __syncthreads();  // tile `it` consumed: its buffer takes tile it + 2
    if (it + 2 < ntiles) issue(it + 2, buf);
  }
#pragma unroll
  for (int o_ = 1; o_ <= 2; o_ <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o_);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o_);
  }
  const float inv0 = l0 > 0.0f ? 1.0f / l0 : 0.0f, inv1 = l1 > 0.0f ? 1.0f / l1 : 0.0f;
  const int r0 = qw + g, r1 = qw + g + 8;
  const int64_t ld = (int64_t)H * kHD;
#pragma unroll
  for (int dt = 0; dt < 8; ++dt) {
    const int c = h * kHD + dt * 8 + 2 * t;
    if (r0 < S)
      *reinterpret_cast<uint32_t*>(out + ((int64_t)b * S + r0) * ld + c) = pack_bf16(o[dt][0] * inv0, o[dt][1] * inv0);
    if (r1 < S)
      *reinterpret_cast<uint32_t*>(out + ((int64_t)b * S + r1) * ld + c) = pack_bf16(o[dt][2] * inv1, o[dt][3] * inv1);
  }
}

// ----------------------------------------------------------------------------- decode attention

// Single-token (decode) attention, split over the context: a CTA handles one
// (batch, KV head, chunk of 128 keys) for the NREP query heads sharing that
// KV head (the NREP heads are the 16 rows of an mma.sync tile, rows past
// NREP are zero), so each cached key / value row is read once per step and a
// 640-token context at batch 64 spreads over 640 CTAs.  The chunk's K and V
// rows stream into shared memory with coalesced cp.async copies (rows past
// the context zero-filled); warp w then takes keys 32w .. 32w+31:
//   S = Q K^T (mma.sync m16n8k16, fp32), the warp's row max m, P = exp2(S -
//   m) rounded to bf16 for P V (as the prefill kernel and the reference's
//   fused kernel do), l = sum of the unrounded P, O = P V (mma.sync);
// the 4 warps' partials merge in shared memory, the chunk's (O, m, l) goes to
// the workspace and attn_decode_combine_kernel merges the chunks of a head.
constexpr int kDecChunk = 128;

// CLUSTER: the nchunks (<= 8) CTAs of one (batch, KV head) form a cluster;
// each sends its chunk partial into CTA 0's shared memory and CTA 0 merges
// them (the combine kernel's arithmetic, chunks in order) straight into `out`.
template <int NREP, bool CLUSTER = false>
__global__ void __launch_bounds__(128) attn_decode_split_kernel(const bf16* __restrict__ q, const bf16* __restrict__ kc,
                                                                const bf16* __restrict__ vc, float* __restrict__ ws,
                                                                int H, int KVH, int smax, int total, int nchunks,
                                                                float scale_log2, bf16* __restrict__ out) {
  static_assert(NREP >= 1 && NREP <= 16, "query heads per KV head fill one 16-row tile");
  __shared__ __align__(16) bf16 sK[kDecChunk][kPad];
  __shared__ __align__(16) bf16 sV[kDecChunk][kPad];
  const int b = blockIdx.x, kvh = blockIdx.y, chunk = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int k0 = chunk * kDecChunk;
  const int nk = min(kDecChunk, total - k0);
  const bf16* kp = kc + ((int64_t)(b * KVH + kvh) * smax + k0) * kHD;
  const bf16* vp = vc + ((int64_t)(b * KVH + kvh) * smax + k0) * kHD;
  const bf16* qp = q + ((int64_t)b * H + kvh * NREP) * kHD;
  pdl_wait();
  pdl_trigger();
#pragma unroll
  for (int j = 0; j < kDecChunk * kHD / 8 / 128; ++j) {
    const int i = tid + 128 * j;
    const int r = i >> 3, c8 = (i & 7) * 8;
    const int src_row = r < nk ? r : 0;     // rows past the context: zero-fill, nothing read
    const uint32_t bytes = r < nk ? 16u : 0u;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                     (uint32_t)__cvta_generic_to_shared(&sK[r][c8])),
                 "l"(kp + (int64_t)src_row * kHD + c8), "r"(bytes)
                 : "memory");
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                     (uint32_t)__cvta_generic_to_shared(&sV[r][c8])),
                 "l"(vp + (int64_t)src_row * kHD + c8), "r"(bytes)
                 : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  uint32_t qa[4][4];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const int c = kk * 16 + 2 * t;
    qa[kk][0] = g < NREP ? *reinterpret_cast<const uint32_t*>(qp + g * kHD + c) : 0u;
    qa[kk][1] = g + 8 < NREP ? *reinterpret_cast<const uint32_t*>(qp + (g + 8) * kHD + c) : 0u;
    qa[kk][2] = g < NREP ? *reinterpret_cast<const uint32_t*>(qp + g * kHD + c + 8) : 0u;
    qa[kk][3] = g + 8 < NREP ? *reinterpret_cast<const uint32_t*>(qp + (g + 8) * kHD + c + 8) : 0u;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();

  const int kw = warp * 32;  // this warp's first key of the chunk
  float sc[4][4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&sK[kw + nt * 8 + g][kk * 16 + 2 * t]);
      const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&sK[kw + nt * 8 + g][kk * 16 + 8 + 2 * t]);
      mma_bf16_16816(sc[nt], qa[kk], b0, b1);
    }
  }
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const bool ok = kw + nt * 8 + 2 * t + (e & 1) < nk;
      sc[nt][e] = ok ? sc[nt][e] * scale_log2 : -INFINITY;
      if (e < 2) mx0 = fmaxf(mx0, sc[nt][e]);
      else mx1 = fmaxf(mx1, sc[nt][e]);
    }
#pragma unroll
  for (int o_ = 1; o_ <= 2; o_ <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o_));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o_));
  }
  const float base0 = mx0 == -INFINITY ? 0.0f : mx0, base1 = mx1 == -INFINITY ? 0.0f : mx1;
  float l0 = 0.0f, l1 = 0.0f;
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    sc[nt][0] = ex2_approx(sc[nt][0] - base0);
    sc[nt][1] = ex2_approx(sc[nt][1] - base0);
    sc[nt][2] = ex2_approx(sc[nt][2] - base1);
    sc[nt][3] = ex2_approx(sc[nt][3] - base1);
    l0 += sc[nt][0] + sc[nt][1];
    l1 += sc[nt][2] + sc[nt][3];
  }
#pragma unroll
  for (int o_ = 1; o_ <= 2; o_ <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o_);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o_);
  }
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {  // keys kw + kk*16 .. kw + kk*16 + 15
    uint32_t pa[4];
    pa[0] = pack_bf16(sc[2 * kk][0], sc[2 * kk][1]);
    pa[1] = pack_bf16(sc[2 * kk][2], sc[2 * kk][3]);
    pa[2] = pack_bf16(sc[2 * kk + 1][0], sc[2 * kk + 1][1]);
    pa[3] = pack_bf16(sc[2 * kk + 1][2], sc[2 * kk + 1][3]);
#pragma unroll
    for (int dt = 0; dt < 8; dt += 2) {
      const int mi = lane >> 3, r = lane & 7;
      uint32_t vb[4];
      ldmatrix_x4_trans(vb, &sV[kw + kk * 16 + (mi & 1) * 8 + r][dt * 8 + (mi >> 1) * 8]);
      mma_bf16_16816(o[dt], pa, vb[0], vb[1]);
      mma_bf16_16816(o[dt + 1], pa, vb[2], vb[3]);
    }
  }
  // Merge the 4 warps' partials of the chunk (max-rescaled sums, warps in
  // order) so the chunk leaves one (O, m, l) per head; the K buffer is free
  // once every warp is past its P V products.
  __shared__ float wm[4][16], wl[4][16];
  if (t == 0) {
    wm[warp][g] = mx0;
    wm[warp][g + 8] = mx1;
    wl[warp][g] = l0;
    wl[warp][g + 8] = l1;
  }
  __syncthreads();
  float* red = reinterpret_cast<float*>(&sK[0][0]);  // [4][16][64] fp32
  static_assert(4 * 16 * kHD * sizeof(float) <= sizeof(sK), "merge buffer fits the K tile");
  auto row_max = [&](int r) {
    return fmaxf(fmaxf(wm[0][r], wm[1][r]), fmaxf(wm[2][r], wm[3][r]));
  };
  {
    const float M0 = row_max(g), M1 = row_max(g + 8);
    const float f0 = ex2_approx(mx0 - (M0 == -INFINITY ? 0.0f : M0));
    const float f1 = ex2_approx(mx1 - (M1 == -INFINITY ? 0.0f : M1));
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) {
      const int d = dt * 8 + 2 * t;
      red[(warp * 16 + g) * kHD + d] = o[dt][0] * f0;
      red[(warp * 16 + g) * kHD + d + 1] = o[dt][1] * f0;
      red[(warp * 16 + g + 8) * kHD + d] = o[dt][2] * f1;
      red[(warp * 16 + g + 8) * kHD + d + 1] = o[dt][3] * f1;
    }
  }
  __syncthreads();
  float pv[(NREP * kHD + 127) / 128];
#pragma unroll
  for (int j = 0; j < (NREP * kHD + 127) / 128; ++j) {
    const int i = tid + 128 * j, r = i / kHD, d = i % kHD;
    pv[j] = i < NREP * kHD ? ((red[r * kHD + d] + red[(16 + r) * kHD + d]) + red[(32 + r) * kHD + d]) +
                                 red[(48 + r) * kHD + d]
                           : 0.0f;
  }
  float pm = 0.0f, pl = 0.0f;
  if (tid < NREP) {
    pm = row_max(tid);
    const float base = pm == -INFINITY ? 0.0f : pm;
#pragma unroll
    for (int w = 0; w < 4; ++w) pl += wl[w][tid] * ex2_approx(wm[w][tid] - base);
  }
  if constexpr (!CLUSTER) {
    float* part = ws + ((int64_t)(b * KVH + kvh) * nchunks + chunk) * NREP * (kHD + 2);
#pragma unroll
    for (int j = 0; j < (NREP * kHD + 127) / 128; ++j) {
      const int i = tid + 128 * j;
      if (i < NREP * kHD) part[(i / kHD) * (kHD + 2) + i % kHD] = pv[j];
    }
    if (tid < NREP) {
      part[tid * (kHD + 2) + kHD] = pm;
      part[tid * (kHD + 2) + kHD + 1] = pl;
    }
  } else {
    static_assert(8 * NREP * (kHD + 2) * sizeof(float) <= sizeof(sK), "8 chunk partials fit CTA 0's K tile");
    float* slots = reinterpret_cast<float*>(&sK[0][0]);  // [nchunks][NREP][kHD + 2] in CTA 0
    xb::tc::cluster_sync();  // every CTA is past its own K tile: CTA 0's may be overwritten
    const uint32_t base = xb::tc::mapa_u32(xb::tc::smem_u32(slots), 0) +
                          (uint32_t)(chunk * NREP * (kHD + 2)) * (uint32_t)sizeof(float);
#pragma unroll
    for (int j = 0; j < (NREP * kHD + 127) / 128; ++j) {
      const int i = tid + 128 * j;
      if (i < NREP * kHD) {
        const uint32_t a = base + (uint32_t)((i / kHD) * (kHD + 2) + i % kHD) * 4u;
        asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(a), "f"(pv[j]) : "memory");
      }
    }
    if (tid < NREP) {
      const uint32_t a = base + (uint32_t)(tid * (kHD + 2) + kHD) * 4u;
      asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(a), "f"(pm) : "memory");
      asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(a + 4u), "f"(pl) : "memory");
    }
    xb::tc::cluster_sync();  // all partials landed in CTA 0; nobody touches a peer afterwards
    if (chunk == 0) {
      for (int i = tid; i < NREP * kHD; i += 128) {
        const int r = i / kHD, d = i % kHD;
        float mx = -INFINITY;
        for (int c = 0; c < nchunks; ++c) mx = fmaxf(mx, slots[(c * NREP + r) * (kHD + 2) + kHD]);
        float l = 0.0f, o = 0.0f;
        for (int c = 0; c < nchunks; ++c) {
          const float* sl = slots + (c * NREP + r) * (kHD + 2);
          const float w = ex2_approx(sl[kHD] - mx);
          l += sl[kHD + 1] * w;
          o += sl[d] * w;
        }
        out[((int64_t)b * H + kvh * NREP + r) * kHD + d] = __float2bfloat16_rn(o / l);
      }
    }
  }
}

// Many sequences, one token each: a CTA per (batch, KV head).  The NREP query
// heads sharing the KV head are the rows of one mma.sync tile; warp w walks
// the 32-key tiles w, w + 8, w + 16, ... of the context with an online
// softmax (P = exp2(S - running max) rounded to bf16 for P V, fp32 l and O
// rescaled when the max grows), double-buffering its own tiles in shared
// memory with cp.async (rows past the context zero-filled), and the eight
// warps' (O, m, l) merge in shared memory in warp order at the end.  The
// context is read once and no cross-CTA merge or second kernel is needed;
// from 48 (batch, KV head) pairs up it beats the chunked kernels (measured:
// 64 pairs 5.3 vs 6.4 us at a 576-key context; 16 pairs 5.3 vs 4.5 us).
// warps per CTA (build-time knob): 8 keeps two of a warp's 32-key tiles in
// flight; 12 puts every tile of a context of up to 768 keys in flight at once
#ifndef XB_HEAD_WARPS
#define XB_HEAD_WARPS 8
#endif
constexpr int kHeadWarps = XB_HEAD_WARPS;
constexpr int kTileK = 32;
constexpr int kHeadTileElems = kTileK * kPad;  // one K or V tile (bf16 elements)
constexpr int kHeadSmem = kHeadWarps * 2 * 2 * kHeadTileElems * (int)sizeof(bf16);

template <int NREP>
__global__ void __launch_bounds__(kHeadWarps * 32, 1) attn_decode_head_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ kc, const bf16* __restrict__ vc, int H, int KVH, int smax,
    int total, float scale_log2, bf16* __restrict__ out) {
  static_assert(NREP >= 1 && NREP <= 16, "query heads per KV head fill one 16-row tile");
  static_assert(kHeadWarps * 16 * kHD * (int)sizeof(float) <= kHeadSmem, "merge buffer fits the tiles");
  extern __shared__ __align__(16) uint8_t head_smem[];
  __shared__ float wm[kHeadWarps][16], wl[kHeadWarps][16];
  const int b = blockIdx.x, kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  bf16* wb = reinterpret_cast<bf16*>(head_smem) + warp * (2 * 2 * kHeadTileElems);
  const bf16* kp = kc + (int64_t)(b * KVH + kvh) * smax * kHD;
  const bf16* vp = vc + (int64_t)(b * KVH + kvh) * smax * kHD;
  const bf16* qp = q + ((int64_t)b * H + kvh * NREP) * kHD;
  const int ntiles = (total + kTileK - 1) / kTileK;
  pdl_wait();
  pdl_trigger();
  // tile `tile` -> buffer `buf` of this warp: 32 keys x 128 bytes of K and of V,
  // 16 bytes per lane per copy, rows past the context zero-filled
  auto issue = [&](int tile, int buf) {
    bf16* sk = wb + (buf * 2) * kHeadTileElems;
    bf16* sv = sk + kHeadTileElems;
#pragma unroll
    for (int j = 0; j < kTileK * kHD / 8 / 32; ++j) {
      const int i = lane + 32 * j;
      const int r = i >> 3, c8 = (i & 7) * 8;
      const int key = tile * kTileK + r;
      const int src = key < total ? key : 0;
      const uint32_t bytes = key < total ? 16u : 0u;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                       (uint32_t)__cvta_generic_to_shared(sk + r * kPad + c8)),
                   "l"(kp + (int64_t)src * kHD + c8), "r"(bytes)
                   : "memory");
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                       (uint32_t)__cvta_generic_to_shared(sv + r * kPad + c8)),
                   "l"(vp + (int64_t)src * kHD + c8), "r"(bytes)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if (warp < ntiles) issue(warp, 0);
  if (warp + kHeadWarps < ntiles) issue(warp + kHeadWarps, 1);
  uint32_t qa[4][4];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const int c = kk * 16 + 2 * t;
    qa[kk][0] = g < NREP ? *reinterpret_cast<const uint32_t*>(qp + g * kHD + c) : 0u;
    qa[kk][1] = g + 8 < NREP ? *reinterpret_cast<const uint32_t*>(qp + (g + 8) * kHD + c) : 0u;
    qa[kk][2] = g < NREP ? *reinterpret_cast<const uint32_t*>(qp + g * kHD + c + 8) : 0u;
    qa[kk][3] = g + 8 < NREP ? *reinterpret_cast<const uint32_t*>(qp + (g + 8) * kHD + c + 8) : 0u;
  }
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  for (int it = 0, tile = warp; tile < ntiles; ++it, tile += kHeadWarps) {
    const int buf = it & 1;
    if (tile + kHeadWarps < ntiles) asm volatile("cp.async.wait_group 1;" ::: "memory");
    else asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncwarp();
    const bf16* sk = wb + (buf * 2) * kHeadTileElems;
    const bf16* sv = sk + kHeadTileElems;
    float s[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(sk + (nt * 8 + g) * kPad + kk * 16 + 2 * t);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(sk + (nt * 8 + g) * kPad + kk * 16 + 8 + 2 * t);
        mma_bf16_16816(s[nt], qa[kk], b0, b1);
      }
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const bool ok = tile * kTileK + nt * 8 + 2 * t + (e & 1) < total;
        s[nt][e] = ok ? s[nt][e] * scale_log2 : -INFINITY;
        if (e < 2) mx0 = fmaxf(mx0, s[nt][e]);
        else mx1 = fmaxf(mx1, s[nt][e]);
      }
#pragma unroll
    for (int o_ = 1; o_ <= 2; o_ <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o_));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o_));
    }
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float base0 = mn0 == -INFINITY ? 0.0f : mn0, base1 = mn1 == -INFINITY ? 0.0f : mn1;
    const float al0 = ex2_approx(m0 - base0), al1 = ex2_approx(m1 - base1);
    m0 = mn0;
    m1 = mn1;
    float rs0 = 0.0f, rs1 = 0.0f;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      s[nt][0] = ex2_approx(s[nt][0] - base0);
      s[nt][1] = ex2_approx(s[nt][1] - base0);
      s[nt][2] = ex2_approx(s[nt][2] - base1);
      s[nt][3] = ex2_approx(s[nt][3] - base1);
      rs0 += s[nt][0] + s[nt][1];
      rs1 += s[nt][2] + s[nt][3];
    }
    l0 = l0 * al0 + rs0;
    l1 = l1 * al1 + rs1;
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) {
      o[dt][0] *= al0;
      o[dt][1] *= al0;
      o[dt][2] *= al1;
      o[dt][3] *= al1;
    }
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {  // keys kk*16 .. kk*16+15 of the tile
      uint32_t pa[4];
      pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dt = 0; dt < 8; dt += 2) {
        const int mi = lane >> 3, r = lane & 7;
        uint32_t vb[4];
        ldmatrix_x4_trans(vb, sv + (kk * 16 + (mi & 1) * 8 + r) * kPad + dt * 8 + (mi >> 1) * 8);
        mma_bf16_16816(o[dt], pa, vb[0], vb[1]);
        mma_bf16_16816(o[dt + 1], pa, vb[2], vb[3]);
      }
    }
    __syncwarp();  // the buffer is free for the tile two steps ahead
    if (tile + 2 * kHeadWarps < ntiles) issue(tile + 2 * kHeadWarps, buf);
  }
#pragma unroll
  for (int o_ = 1; o_ <= 2; o_ <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o_);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o_);
  }
  if (t == 0) {
    wm[warp][g] = m0;
    wm[warp][g + 8] = m1;
    wl[warp][g] = l0;
    wl[warp][g + 8] = l1;
  }
  __syncthreads();  // every warp is past its tiles: the buffers hold the merge
  float* red = reinterpret_cast<float*>(head_smem);  // [warp][16][64] fp32
  {
    float M0 = -INFINITY, M1 = -INFINITY;
#pragma unroll
    for (int w = 0; w < kHeadWarps; ++w) {
      M0 = fmaxf(M0, wm[w][g]);
      M1 = fmaxf(M1, wm[w][g + 8]);
    }
    const float f0 = m0 == -INFINITY ? 0.0f : ex2_approx(m0 - M0);
    const float f1 = m1 == -INFINITY ? 0.0f : ex2_approx(m1 - M1);
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) {
      const int d = dt * 8 + 2 * t;
      red[(warp * 16 + g) * kHD + d] = o[dt][0] * f0;
      red[(warp * 16 + g) * kHD + d + 1] = o[dt][1] * f0;
      red[(warp * 16 + g + 8) * kHD + d] = o[dt][2] * f1;
      red[(warp * 16 + g + 8) * kHD + d + 1] = o[dt][3] * f1;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < NREP * kHD; i += kHeadWarps * 32) {
    const int r = i / kHD, d = i % kHD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kHeadWarps; ++w) M = fmaxf(M, wm[w][r]);
    float acc = 0.0f, l = 0.0f;
#pragma unroll
    for (int w = 0; w < kHeadWarps; ++w) {
      acc += red[(w * 16 + r) * kHD + d];
      l += wm[w][r] == -INFINITY ? 0.0f : wl[w][r] * ex2_approx(wm[w][r] - M);
    }
    out[((int64_t)b * H + kvh * NREP + r) * kHD + d] = __float2bfloat16_rn(acc / l);
  }
}

// The same partials computed on the CUDA cores, for one or two query heads
// per KV head (GPT-2's multi-head attention), where a 16-row mma tile would
// be mostly padding: thread t scores key t of the chunk (K rows staged in
// shared memory, padded for conflict-free 16-byte reads), warps reduce the
// chunk max and sum, warp w accumulates P V over keys 32w .. 32w+31.
template <int NREP>
__global__ void __launch_bounds__(128) attn_decode_scalar_kernel(const bf16* __restrict__ q, const bf16* __restrict__ kc,
                                                                const bf16* __restrict__ vc, float* __restrict__ ws,
                                                                int H, int KVH, int smax, int total, int nchunks,
                                                                float scale_log2) {
  // K rows are padded to 72 elements (144 bytes) so thread t reading row t
  // with 16-byte loads is bank-conflict free; the P@V partial sums reuse the
  // K buffer once the scores are done.
  constexpr int kKPad = kHD + 8;
  __shared__ __align__(16) bf16 vs[kDecChunk][kHD];
  __shared__ __align__(16) bf16 ks[kDecChunk * kKPad];
  __shared__ float qs[NREP][kHD];
  __shared__ float ps[NREP][kDecChunk];
  __shared__ float stat[NREP][2];
  static_assert(4 * NREP * kHD * sizeof(float) <= sizeof(ks), "partial sums fit the K buffer");
  float(*red)[NREP][kHD] = reinterpret_cast<float(*)[NREP][kHD]>(ks);
  const int b = blockIdx.x, kvh = blockIdx.y, chunk = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int k0 = chunk * kDecChunk;
  const int nk = min(kDecChunk, total - k0);
  const bf16* kp = kc + ((int64_t)(b * KVH + kvh) * smax + k0) * kHD;
  const bf16* vp = vc + ((int64_t)(b * KVH + kvh) * smax + k0) * kHD;
  pdl_wait();
  pdl_trigger();
  // Every global load of the CTA is issued up front with coalesced 16-byte
  // cp.async copies (consecutive threads, consecutive addresses): the K chunk
  // (group 0), the V chunk (group 1), then q.
#pragma unroll
  for (int j = 0; j < kDecChunk * kHD / 8 / 128; ++j) {
    const int i = tid + 128 * j;
    const int r = i >> 3, c8 = (i & 7) * 8;
    if (r < nk)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                       (uint32_t)__cvta_generic_to_shared(&ks[r * kKPad + c8])),
                   "l"(kp + (int64_t)r * kHD + c8)
                   : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
#pragma unroll
  for (int j = 0; j < kDecChunk * kHD / 8 / 128; ++j) {
    const int i = tid + 128 * j;
    const int r = i >> 3, c8 = (i & 7) * 8;
    if (r < nk)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(&vs[r][c8])),
                   "l"(vp + (int64_t)r * kHD + c8)
                   : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int i = tid; i < NREP * kHD; i += 128)
    qs[i / kHD][i % kHD] = __bfloat162float(q[((int64_t)b * H + kvh * NREP + i / kHD) * kHD + i % kHD]);
  asm volatile("cp.async.wait_group 1;" ::: "memory");  // this thread's K copies have landed
  __syncthreads();
  int4 kr[kHD / 8];
  if (tid < nk) {
#pragma unroll
    for (int c = 0; c < kHD / 8; ++c) kr[c] = *reinterpret_cast<const int4*>(&ks[tid * kKPad + c * 8]);
  }

  if (tid < nk) {
    float acc[NREP];
#pragma unroll
    for (int r = 0; r < NREP; ++r) acc[r] = 0.0f;
#pragma unroll
    for (int c = 0; c < kHD / 8; ++c) {
      const __nv_bfloat162* kv = reinterpret_cast<const __nv_bfloat162*>(&kr[c]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float kx = __low2float(kv[e]), ky = __high2float(kv[e]);
#pragma unroll
        for (int r = 0; r < NREP; ++r) {
          const float2 qq = *reinterpret_cast<const float2*>(&qs[r][c * 8 + 2 * e]);
          acc[r] += qq.x * kx + qq.y * ky;
        }
      }
    }
#pragma unroll
    for (int r = 0; r < NREP; ++r) ps[r][tid] = acc[r] * scale_log2;
  } else {
#pragma unroll
    for (int r = 0; r < NREP; ++r) ps[r][tid] = -INFINITY;
  }
  __syncthreads();
  for (int r = warp; r < NREP; r += 4) {
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kDecChunk / 32; ++j) mx = fmaxf(mx, ps[r][lane + 32 * j]);
#pragma unroll
    for (int o_ = 16; o_ > 0; o_ >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o_));
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < kDecChunk / 32; ++j) {
      const int k = lane + 32 * j;
      const float p = k < nk ? ex2_approx(ps[r][k] - mx) : 0.0f;
      sum += p;
      ps[r][k] = __bfloat162float(__float2bfloat16_rn(p));
    }
#pragma unroll
    for (int o_ = 16; o_ > 0; o_ >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o_);
    if (lane == 0) {
      stat[r][0] = mx;
      stat[r][1] = sum;
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();  // V landed; every thread is past its K reads (red reuses ks)
  float ax[NREP], ay[NREP];
#pragma unroll
  for (int r = 0; r < NREP; ++r) ax[r] = ay[r] = 0.0f;
  const int kend = min(32 * warp + 32, nk);
#pragma unroll 8
  for (int k = 32 * warp; k < kend; ++k) {
    const __nv_bfloat162 vv = *reinterpret_cast<const __nv_bfloat162*>(&vs[k][2 * lane]);
    const float vx = __low2float(vv), vy = __high2float(vv);
#pragma unroll
    for (int r = 0; r < NREP; ++r) {
      const float p = ps[r][k];
      ax[r] += p * vx;
      ay[r] += p * vy;
    }
  }
#pragma unroll
  for (int r = 0; r < NREP; ++r) {
    red[warp][r][2 * lane] = ax[r];
    red[warp][r][2 * lane + 1] = ay[r];
  }
  __syncthreads();
  float* part = ws + ((int64_t)(b * KVH + kvh) * nchunks + chunk) * NREP * (kHD + 2);
  for (int i = tid; i < NREP * kHD; i += 128) {
    const int r = i / kHD, d = i % kHD;
    part[r * (kHD + 2) + d] = red[0][r][d] + red[1][r][d] + red[2][r][d] + red[3][r][d];
  }
  if (tid < NREP) {
    part[tid * (kHD + 2) + kHD] = stat[tid][0];
    part[tid * (kHD + 2) + kHD + 1] = stat[tid][1];
  }
}

// out[b, h, :] = sum_c o_c 2^(m_c - M) / sum_c l_c 2^(m_c - M), M = max_c m_c.
__global__ void __launch_bounds__(kHD) attn_decode_combine_kernel(const float* __restrict__ ws, bf16* __restrict__ out,
                                                                  int H, int KVH, int nchunks) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int n_rep = H / KVH;
  const int kvh = h / n_rep, r = h % n_rep;
  const float* base = ws + ((int64_t)(b * KVH + kvh) * nchunks) * n_rep * (kHD + 2) + r * (kHD + 2);
  const int64_t cstride = (int64_t)n_rep * (kHD + 2);
  float mx = -INFINITY;
  for (int c = 0; c < nchunks; ++c) mx = fmaxf(mx, base[c * cstride + kHD]);
  float l = 0.0f, o = 0.0f;
  for (int c = 0; c < nchunks; ++c) {
    const float w = ex2_approx(base[c * cstride + kHD] - mx);
    l += base[c * cstride + kHD + 1] * w;
    o += base[c * cstride + d] * w;
  }
  out[((int64_t)b * H + h) * kHD + d] = __float2bfloat16_rn(o / l);
}

// ----------------------------------------------------------------------------- argmax

__device__ __forceinline__ bool better(float v1, int64_t i1, float v2, int64_t i2, int64_t cols) {
  return xb::argmax_better(v1, i1, v2, i2, cols);
}

// idx[r] = first index of the maximum of logits[r, :].
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ x, int64_t cols, int64_t ld,
                                                      int64_t* __restrict__ idx) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sv[32];
  __shared__ int64_t si[32];
  const float* row = x + (int64_t)blockIdx.x * ld;
  float best = 0.0f;
  int64_t bi = cols;
  // 16-byte loads, four in flight per thread, when the row allows it; each
  // thread still visits its indices in increasing order, so ties keep the
  // first index.
  int64_t vec_end = 0;
  if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    vec_end = cols / 4 * 4;
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const int64_t n4 = vec_end / 4;
    for (int64_t base = threadIdx.x; base < n4; base += 4 * (int64_t)blockDim.x) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t i = base + (int64_t)u * blockDim.x;
        v[u] = i < n4 ? __ldcs(r4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t i = base + (int64_t)u * blockDim.x;
        if (i < n4) {
          const float e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (better(best, bi, e[j], 4 * i + j, cols)) {
              best = e[j];
              bi = 4 * i + j;
            }
        }
      }
    }
  }
  for (int64_t c = vec_end + threadIdx.x; c < cols; c += blockDim.x) {
    const float v = row[c];
    if (better(best, bi, v, c, cols)) {
      best = v;
      bi = c;
    }
  }
#pragma unroll
  for (int o_ = 16; o_ > 0; o_ >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o_);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o_);
    if (better(best, bi, ov, oi, cols)) {
      best = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = (blockDim.x + 31) / 32;
    best = lane < nw ? sv[lane] : 0.0f;
    bi = lane < nw ? si[lane] : cols;
#pragma unroll
    for (int o_ = 16; o_ > 0; o_ >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o_);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o_);
      if (better(best, bi, ov, oi, cols)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) idx[blockIdx.x] = bi < cols ? bi : 0;
  }
}

__device__ int g_bad_token = 0;

}  // namespace llm
}  // namespace xb

using namespace xb::llm;
using xb::set_err;
using xb::check_launch;
using xb::launch_k;

extern "C" int xb_embedding_bf16(const void* table, const int64_t* ids, void* out, int64_t rows, int64_t dim,
                                 int64_t vocab, void* stream, char* err, size_t errlen) {
  if (rows < 0 || dim <= 0 || vocab <= 0) {
    set_err(err, errlen, "xb_embedding_bf16: bad shape");
    return XB_ERR_INVALID;
  }
  if (rows == 0) return XB_OK;
  if (!table || !ids || !out) {
    set_err(err, errlen, "xb_embedding_bf16: null pointer");
    return XB_ERR_INVALID;
  }
  if (dim % 8 || !xb::aligned16(table) || !xb::aligned16(out)) {
    set_err(err, errlen, "xb_embedding_bf16: rows must be whole 16-byte vectors (dim %% 8 == 0, aligned)");
    return XB_ERR_UNSUPPORTED;
  }
  int* bad = nullptr;
  if (cudaGetSymbolAddress((void**)&bad, g_bad_token) != cudaSuccess) {
    set_err(err, errlen, "xb_embedding_bf16: status word unavailable");
    return XB_ERR_CUDA;
  }
  launch_k<false>(embedding_kernel, (unsigned)((rows + 7) / 8), 256, 0, (cudaStream_t)stream, static_cast<const bf16*>(table),
           ids, static_cast<bf16*>(out), rows, dim, vocab, bad);
  return check_launch("xb_embedding_bf16", err, errlen);
}

extern "C" int xb_token_status(void* stream, int* status, char* err, size_t errlen) {
  if (!status) {
    set_err(err, errlen, "xb_token_status: null output");
    return XB_ERR_INVALID;
  }
  cudaStream_t s = (cudaStream_t)stream;
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(status, g_bad_token, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(g_bad_token, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    set_err(err, errlen, "xb_token_status: %s", cudaGetErrorString(e));
    return XB_ERR_CUDA;
  }
  return XB_OK;
}

extern "C" int xb_embedding_pos_bf16(const void* table, const void* pos_table, const int64_t* ids, void* out,
                                     int64_t rows, int64_t seq, int64_t dim, int64_t vocab, int64_t n_pos,
                                     int64_t pos_offset, void* stream, char* err, size_t errlen) {
  const char* what = "xb_embedding_pos_bf16";
  if (rows < 0 || seq <= 0 || dim <= 0 || vocab <= 0 || n_pos <= 0 || pos_offset < 0 || (rows % seq) != 0) {
    set_err(err, errlen, "%s: bad shape", what);
    return XB_ERR_INVALID;
  }
  if (pos_offset + seq > n_pos) {
    set_err(err, errlen, "%s: positions %lld..%lld exceed the position table (%lld)", what, (long long)pos_offset,
            (long long)(pos_offset + seq - 1), (long long)n_pos);
    return XB_ERR_INVALID;
  }
  if (rows == 0) return XB_OK;
  if (!table || !pos_table || !ids || !out) {
    set_err(err, errlen, "%s: null pointer", what);
    return XB_ERR_INVALID;
  }
  if (dim % 8 || !xb::aligned16(table) || !xb::aligned16(pos_table) || !xb::aligned16(out)) {
    set_err(err, errlen, "%s: rows must be whole 16-byte vectors (dim %% 8 == 0, aligned)", what);
    return XB_ERR_UNSUPPORTED;
  }
  int* bad = nullptr;
  if (cudaGetSymbolAddress((void**)&bad, g_bad_token) != cudaSuccess) {
    set_err(err, errlen, "%s: status word unavailable", what);
    return XB_ERR_CUDA;
  }
  launch_k<false>(embedding_pos_kernel, (unsigned)((rows + 7) / 8), 256, 0, (cudaStream_t)stream,
           static_cast<const bf16*>(table), static_cast<const bf16*>(pos_table), ids, static_cast<bf16*>(out), rows,
           dim, vocab, (int)seq, (int)pos_offset, bad);
  return check_launch(what, err, errlen);
}

extern "C" int xb_rope_kv_bf16(const void* qkv, const float* cos_t, const float* sin_t, void* q_out, void* k_cache,
                               void* v_cache, int64_t batch, int64_t seq, int64_t n_head, int64_t n_kv_head,
                               int64_t head_dim, int64_t max_seq, int64_t pos_offset, void* stream, char* err,
                               size_t errlen) {
  if (batch < 0 || seq < 0 || n_head <= 0 || n_kv_head <= 0 || head_dim <= 0 || head_dim % 2 || pos_offset < 0 ||
      n_head % n_kv_head) {
    set_err(err, errlen, "xb_rope_kv_bf16: bad shape");
    return XB_ERR_INVALID;
  }
  if (pos_offset + seq > max_seq) {
    set_err(err, errlen, "xb_rope_kv_bf16: positions %lld..%lld exceed the cache (%lld)", (long long)pos_offset,
            (long long)(pos_offset + seq - 1), (long long)max_seq);
    return XB_ERR_INVALID;
  }
  if (batch == 0 || seq == 0) return XB_OK;
  if (!qkv || !q_out || !k_cache || !v_cache || (!cos_t) != (!sin_t)) {
    set_err(err, errlen, "xb_rope_kv_bf16: null pointer");
    return XB_ERR_INVALID;
  }
  const int64_t per_token = (n_head + 2 * n_kv_head) * (head_dim / 2);
  const int threads = per_token >= 1024 ? 1024 : (int)((per_token + 31) / 32 * 32);
  if (batch * seq > 0x7fffffffLL) {
    set_err(err, errlen, "xb_rope_kv_bf16: too many tokens");
    return XB_ERR_UNSUPPORTED;
  }
  const bool vec = head_dim % 4 == 0 && (reinterpret_cast<uintptr_t>(qkv) & 3) == 0 &&
                   (reinterpret_cast<uintptr_t>(q_out) & 3) == 0 && (reinterpret_cast<uintptr_t>(k_cache) & 3) == 0 &&
                   (reinterpret_cast<uintptr_t>(v_cache) & 3) == 0 &&
                   (!cos_t || ((reinterpret_cast<uintptr_t>(cos_t) & 7) == 0 && (reinterpret_cast<uintptr_t>(sin_t) & 7) == 0));
  if (vec && batch * seq >= 256) {
    const int64_t items = batch * seq * (n_head + 2 * n_kv_head) * (head_dim / 4);
    int64_t grid = (items + 255) / 256;
    int sms = 148;
    xb::sm_count(&sms);
    if (grid > (int64_t)sms * 16) grid = (int64_t)sms * 16;
    launch_k<false>(rope_kv_flat_kernel, (unsigned)grid, 256, 0, (cudaStream_t)stream, static_cast<const bf16*>(qkv),
                    cos_t, sin_t, static_cast<bf16*>(q_out), static_cast<bf16*>(k_cache), static_cast<bf16*>(v_cache),
                    batch * seq, (int)seq, (int)n_head, (int)n_kv_head, (int)head_dim, (int)max_seq, (int)pos_offset);
    return check_launch("xb_rope_kv_bf16", err, errlen);
  }
  launch_k<false>(rope_kv_kernel, (unsigned)(batch * seq), threads, 0, (cudaStream_t)stream, static_cast<const bf16*>(qkv),
           cos_t, sin_t, static_cast<bf16*>(q_out), static_cast<bf16*>(k_cache), static_cast<bf16*>(v_cache), (int)seq,
           (int)n_head, (int)n_kv_head, (int)head_dim, (int)max_seq, (int)pos_offset);
  return check_launch("xb_rope_kv_bf16", err, errlen);
}

// Launch attn_decode_head_kernel<R> (its shared-memory limit raised once).
template <int R>
static cudaError_t launch_head(dim3 grid, cudaStream_t s, const bf16* q, const bf16* k, const bf16* v, int H, int KVH,
                               int smax, int total, float scale_log2, bf16* out) {
  cudaError_t e = xb::once_per_device(reinterpret_cast<const void*>(attn_decode_head_kernel<R>), xb::kOnceSmem, [](int*) {
    return cudaFuncSetAttribute(attn_decode_head_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, kHeadSmem);
  });
  if (e != cudaSuccess) return e;
  return launch_k(attn_decode_head_kernel<R>, grid, kHeadWarps * 32, kHeadSmem, s, q, k, v, H, KVH, smax, total,
                  scale_log2, out);
}

// XB_HEAD_ATTN=0 in the environment keeps many-sequence decode attention on
// the chunked kernels (A/B timing).
static bool head_attn_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("XB_HEAD_ATTN");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

namespace xb {
int attention_prefill_tc(const void* q, const void* k_cache, const void* v_cache, void* out, int64_t batch,
                         int64_t seq, int64_t n_head, int64_t n_kv_head, int64_t max_seq, int64_t pos_offset,
                         float scale_log2, cudaStream_t s, const char* what, char* err, size_t errlen);
}  // namespace xb

// Prefill attention on tcgen05 (csrc/gemm.cu); XB_ATTN_TC=0 in the
// environment selects the mma.sync kernel above (also taken when an operand
// breaks the TMA alignment rules).
static bool attn_tc_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("XB_ATTN_TC");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

extern "C" int xb_attention_workspace_size(int64_t batch, int64_t seq, int64_t n_head, int64_t n_kv_head,
                                           int64_t pos_offset, size_t* bytes, char* err, size_t errlen) {
  if (!bytes || batch < 0 || seq < 0 || n_head <= 0 || n_kv_head <= 0 || pos_offset < 0) {
    set_err(err, errlen, "xb_attention_workspace_size: bad arguments");
    return XB_ERR_INVALID;
  }
  if (seq != 1) {
    *bytes = 0;
    return XB_OK;
  }
  const int64_t nchunks = (pos_offset + 1 + kDecChunk - 1) / kDecChunk;
  *bytes = (size_t)(batch * n_kv_head * nchunks * (n_head / n_kv_head) * (kHD + 2)) * sizeof(float);
  return XB_OK;
}

extern "C" int xb_attention_bf16(const void* q, const void* k_cache, const void* v_cache, void* out, int64_t batch,
                                 int64_t seq, int64_t n_head, int64_t n_kv_head, int64_t head_dim, int64_t max_seq,
                                 int64_t pos_offset, float scale, void* workspace, size_t workspace_bytes,
                                 void* stream, char* err, size_t errlen) {
  const char* what = "xb_attention_bf16";
  if (batch < 0 || seq < 0 || n_head <= 0 || n_kv_head <= 0 || n_head % n_kv_head || pos_offset < 0) {
    set_err(err, errlen, "%s: bad shape", what);
    return XB_ERR_INVALID;
  }
  if (head_dim != kHD) {
    set_err(err, errlen, "%s: head_dim %lld not supported (64)", what, (long long)head_dim);
    return XB_ERR_UNSUPPORTED;
  }
  if (pos_offset + seq > max_seq) {
    set_err(err, errlen, "%s: keys beyond the cache", what);
    return XB_ERR_INVALID;
  }
  if (batch == 0 || seq == 0) return XB_OK;
  if (!q || !k_cache || !v_cache || !out) {
    set_err(err, errlen, "%s: null pointer", what);
    return XB_ERR_INVALID;
  }
  if (batch > 65535 || n_kv_head > 65535 || batch * n_head > 65535) {
    set_err(err, errlen, "%s: grid too large", what);
    return XB_ERR_UNSUPPORTED;
  }
  const float scale_log2 = scale * 1.4426950408889634f;
  cudaStream_t s = (cudaStream_t)stream;
  if (seq == 1) {
    const int total = (int)(pos_offset + 1);
    const int n_rep = (int)(n_head / n_kv_head);
    const int nchunks = (total + kDecChunk - 1) / kDecChunk;
    const size_t need = (size_t)batch * n_kv_head * nchunks * n_rep * (kHD + 2) * sizeof(float);
    if (!workspace || workspace_bytes < need) {
      set_err(err, errlen, "%s: decode needs a workspace of %zu bytes (%zu given)", what, need, workspace_bytes);
      return XB_ERR_INVALID;
    }
    float* ws = static_cast<float*>(workspace);
    dim3 grid((unsigned)batch, (unsigned)n_kv_head, (unsigned)nchunks);
    const bf16* qq = static_cast<const bf16*>(q);
    const bf16* kk = static_cast<const bf16*>(k_cache);
    const bf16* vv = static_cast<const bf16*>(v_cache);
    const int Hh = (int)n_head, KV = (int)n_kv_head, SM = (int)max_seq;
    bf16* ob = static_cast<bf16*>(out);
    // many (batch, KV head) pairs: one CTA each walks the whole context
    if (n_rep >= 3 && n_rep <= 8 && batch * n_kv_head >= 48 && head_attn_enabled()) {
      const dim3 hg((unsigned)batch, (unsigned)n_kv_head);
      cudaError_t ce;
      switch (n_rep) {
        case 3: ce = launch_head<3>(hg, s, qq, kk, vv, Hh, KV, SM, total, scale_log2, ob); break;
        case 4: ce = launch_head<4>(hg, s, qq, kk, vv, Hh, KV, SM, total, scale_log2, ob); break;
        case 5: ce = launch_head<5>(hg, s, qq, kk, vv, Hh, KV, SM, total, scale_log2, ob); break;
        case 6: ce = launch_head<6>(hg, s, qq, kk, vv, Hh, KV, SM, total, scale_log2, ob); break;
        case 7: ce = launch_head<7>(hg, s, qq, kk, vv, Hh, KV, SM, total, scale_log2, ob); break;
        default: ce = launch_head<8>(hg, s, qq, kk, vv, Hh, KV, SM, total, scale_log2, ob); break;
      }
      if (ce != cudaSuccess) {
        set_err(err, errlen, "%s: %s", what, cudaGetErrorString(ce));
        return XB_ERR_CUDA;
      }
      return check_launch(what, err, errlen);
    }
    // contexts of up to 8 chunks merge inside a cluster (no combine launch)
    const bool clustered = n_rep >= 3 && nchunks <= 8;
    auto launch_cluster = [&](auto kernel) -> cudaError_t {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = grid;
      cfg.blockDim = dim3(128);
      cfg.stream = s;
      cudaLaunchAttribute attr[2];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 1;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = (unsigned)nchunks;
      attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[1].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = xb::pdl_enabled() ? 2 : 1;
      xb::prefer_max_smem(reinterpret_cast<const void*>(kernel));
      xb::launch_counter().fetch_add(1, std::memory_order_relaxed);
      return cudaLaunchKernelEx(&cfg, kernel, qq, kk, vv, ws, Hh, KV, SM, total, nchunks, scale_log2, ob);
    };
    cudaError_t ce = cudaSuccess;
    switch (n_rep) {
#define XB_DEC(R)                                                                                              \
  case R:                                                                                                      \
    if (clustered) ce = launch_cluster(attn_decode_split_kernel<R, true>);                                    \
    else launch_k(attn_decode_split_kernel<R>, grid, 128, 0, s, qq, kk, vv, ws, Hh, KV, SM, total, nchunks,    \
                  scale_log2, ob);                                                                             \
    break;
#define XB_DEC_SCALAR(R) \
  case R: launch_k(attn_decode_scalar_kernel<R>, grid, 128, 0, s, qq, kk, vv, ws, Hh, KV, SM, total, nchunks, scale_log2); break;
      XB_DEC_SCALAR(1) XB_DEC_SCALAR(2) XB_DEC(3) XB_DEC(4) XB_DEC(5) XB_DEC(6) XB_DEC(7) XB_DEC(8)
#undef XB_DEC
#undef XB_DEC_SCALAR
      default:
        set_err(err, errlen, "%s: %d query heads per KV head not supported (1..8)", what, n_rep);
        return XB_ERR_UNSUPPORTED;
    }
    if (ce != cudaSuccess) {
      set_err(err, errlen, "%s: %s", what, cudaGetErrorString(ce));
      return XB_ERR_CUDA;
    }
    if (!clustered)
      launch_k(attn_decode_combine_kernel, dim3((unsigned)batch, (unsigned)n_head), kHD, 0, s, (const float*)ws,
               static_cast<bf16*>(out), Hh, KV, nchunks);
  } else {
    if (attn_tc_enabled()) {  // tcgen05 kernel; operands that break its TMA rules take the mma.sync kernel
      const int rc = xb::attention_prefill_tc(q, k_cache, v_cache, out, batch, seq, n_head, n_kv_head, max_seq,
                                              pos_offset, scale_log2, s, what, err, errlen);
      if (rc != XB_ERR_UNSUPPORTED) return rc;
    }
    dim3 grid((unsigned)((seq + kBQ - 1) / kBQ), (unsigned)(batch * n_head));
    launch_k(attn_prefill_kernel, grid, 128, 0, s, static_cast<const bf16*>(q), static_cast<const bf16*>(k_cache),
                                             static_cast<const bf16*>(v_cache), static_cast<bf16*>(out),
                                             (int)n_head, (int)n_kv_head, (int)seq, (int)max_seq, (int)pos_offset,
                                             scale_log2);
  }
  return check_launch(what, err, errlen);
}

// Long rows (the vocabulary logits of a decode step): a cluster of 8 CTAs
// splits each row into 8 column ranges (multiples of 4 columns, 16-byte loads
// when the row is aligned), reduces each range in its CTA, and CTA 0 merges
// the 8 candidates through distributed shared memory.  `better` is a total
// order (value, then smaller index; NaN largest), so the merge order does not
// change the result.
constexpr int kArgmaxSplit = 8;
__global__ void __launch_bounds__(256) argmax_cluster_kernel(const float* __restrict__ x, int64_t cols, int64_t ld,
                                                             int64_t* __restrict__ idx) {
  __shared__ float sv[8];
  __shared__ int64_t si[8];
  __shared__ float cand_v[kArgmaxSplit];
  __shared__ int64_t cand_i[kArgmaxSplit];
  const uint32_t rank = xb::tc::cluster_ctarank();
  xb::pdl_wait();
  xb::pdl_trigger();
  const float* row = x + (int64_t)blockIdx.x * ld;
  const int64_t chunk = ((cols + kArgmaxSplit - 1) / kArgmaxSplit + 3) / 4 * 4;
  const int64_t c0 = min(cols, (int64_t)rank * chunk), c1 = min(cols, c0 + chunk);
  float best = 0.0f;
  int64_t bi = cols;
  int64_t vec_end = c0;
  if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    vec_end = c0 + (c1 - c0) / 4 * 4;
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const int64_t a4 = c0 / 4, n4 = vec_end / 4;
    for (int64_t base = a4 + threadIdx.x; base < n4; base += 4 * (int64_t)blockDim.x) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t i = base + (int64_t)u * blockDim.x;
        v[u] = i < n4 ? __ldcs(r4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t i = base + (int64_t)u * blockDim.x;
        if (i < n4) {
          const float e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (better(best, bi, e[j], 4 * i + j, cols)) {
              best = e[j];
              bi = 4 * i + j;
            }
        }
      }
    }
  }
  for (int64_t c = vec_end + threadIdx.x; c < c1; c += blockDim.x) {
    const float v = row[c];
    if (better(best, bi, v, c, cols)) {
      best = v;
      bi = c;
    }
  }
#pragma unroll
  for (int o_ = 16; o_ > 0; o_ >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o_);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o_);
    if (better(best, bi, ov, oi, cols)) {
      best = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    best = lane < 8 ? sv[lane] : 0.0f;
    bi = lane < 8 ? si[lane] : cols;
#pragma unroll
    for (int o_ = 16; o_ > 0; o_ >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o_);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o_);
      if (better(best, bi, ov, oi, cols)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) {  // this range's candidate into CTA 0's shared memory
      const uint32_t dv = xb::tc::mapa_u32(xb::tc::smem_u32(&cand_v[rank]), 0);
      const uint32_t di = xb::tc::mapa_u32(xb::tc::smem_u32(&cand_i[rank]), 0);
      asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dv), "f"(best) : "memory");
      asm volatile("st.shared::cluster.s64 [%0], %1;" ::"r"(di), "l"(bi) : "memory");
    }
  }
  xb::tc::cluster_sync();  // candidates visible in CTA 0; no CTA touches another's memory afterwards
  if (rank == 0 && threadIdx.x == 0) {
    float b = cand_v[0];
    int64_t i0 = cand_i[0];
    for (int r = 1; r < kArgmaxSplit; ++r)
      if (better(b, i0, cand_v[r], cand_i[r], cols)) {
        b = cand_v[r];
        i0 = cand_i[r];
      }
    idx[blockIdx.x] = i0 < cols ? i0 : 0;
  }
}

extern "C" int xb_argmax_f32(const float* x, int64_t rows, int64_t cols, int64_t ld, int64_t* idx, void* stream,
                             char* err, size_t errlen) {
  if (rows < 0 || cols <= 0 || ld < cols) {
    set_err(err, errlen, "xb_argmax_f32: bad shape");
    return XB_ERR_INVALID;
  }
  if (rows == 0) return XB_OK;
  if (!x || !idx) {
    set_err(err, errlen, "xb_argmax_f32: null pointer");
    return XB_ERR_INVALID;
  }
  if (cols >= 8192 && rows <= 0x7fffffffLL) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)rows, kArgmaxSplit, 1);
    cfg.blockDim = dim3(256);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = kArgmaxSplit;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = xb::pdl_enabled() ? 2 : 1;
    xb::launch_counter().fetch_add(1, std::memory_order_relaxed);
    cudaError_t e = cudaLaunchKernelEx(&cfg, argmax_cluster_kernel, x, cols, ld, idx);
    if (e != cudaSuccess) {
      set_err(err, errlen, "xb_argmax_f32: %s", cudaGetErrorString(e));
      return XB_ERR_CUDA;
    }
    return check_launch("xb_argmax_f32", err, errlen);
  }
  launch_k<false>(argmax_kernel, (unsigned)rows, 1024, 0, (cudaStream_t)stream, x, cols, ld, idx);
  return check_launch("xb_argmax_f32", err, errlen);
}
