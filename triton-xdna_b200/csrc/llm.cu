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

namespace xb {
namespace llm {

typedef __nv_bfloat16 bf16;

// ----------------------------------------------------------------------------- embedding

// out[m, :] = table[ids[m], :]; one warp per row, 16-byte vectors.
__global__ void __launch_bounds__(256) embedding_kernel(const bf16* __restrict__ table, const int64_t* __restrict__ ids,
                                                        bf16* __restrict__ out, int64_t rows, int64_t dim,
                                                        int64_t vocab, int* __restrict__ bad) {
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

// ----------------------------------------------------------------------------- RoPE + KV write

// One thread per (token, head slot, pair i < D/2).  Head slots [0, H) are
// queries, [H, H+KVH) keys, [H+KVH, H+2KVH) values (copied unrotated).
// x_out[i] = x[i]*cos - x[i+D/2]*sin, x_out[i+D/2] = x[i+D/2]*cos + x[i]*sin,
// each product and sum rounded separately in fp32 as rope.py:63-66 does.
__global__ void __launch_bounds__(256) rope_kv_kernel(const bf16* __restrict__ qkv, const float* __restrict__ cos_t,
                                                      const float* __restrict__ sin_t, bf16* __restrict__ q_out,
                                                      bf16* __restrict__ k_cache, bf16* __restrict__ v_cache, int B,
                                                      int S, int H, int KVH, int D, int smax, int pos_offset) {
  const int half = D / 2;
  const int slots = H + 2 * KVH;
  const int64_t total = (int64_t)B * S * slots * half;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(idx % half);
    const int64_t r = idx / half;
    const int slot = (int)(r % slots);
    const int64_t m = r / slots;  // token row b*S + s
    const int s = (int)(m % S);
    const int b = (int)(m / S);
    const bf16* x = qkv + m * (int64_t)(slots * D) + (int64_t)slot * D;
    const int pos = pos_offset + s;
    if (slot >= H + KVH) {  // value head: copy
      const int kh = slot - H - KVH;
      bf16* dst = v_cache + (((int64_t)b * KVH + kh) * smax + pos) * D;
      dst[i] = x[i];
      dst[i + half] = x[i + half];
      continue;
    }
    const float x0 = __bfloat162float(x[i]);
    const float x1 = __bfloat162float(x[i + half]);
    const float c = cos_t[(int64_t)pos * D + i];
    const float sn = sin_t[(int64_t)pos * D + i];
    const float c2 = cos_t[(int64_t)pos * D + i + half];
    const float s2 = sin_t[(int64_t)pos * D + i + half];
    const float y0 = __fadd_rn(__fmul_rn(x0, c), __fmul_rn(-x1, sn));
    const float y1 = __fadd_rn(__fmul_rn(x1, c2), __fmul_rn(x0, s2));
    bf16* dst;
    if (slot < H) {
      dst = q_out + (((int64_t)b * H + slot) * S + s) * D;
    } else {
      dst = k_cache + (((int64_t)b * KVH + (slot - H)) * smax + pos) * D;
    }
    dst[i] = __float2bfloat16_rn(y0);
    dst[i + half] = __float2bfloat16_rn(y1);
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

// Causal GQA attention, FlashAttention-style: a CTA of 4 warps owns 64 query
// rows of one (batch, head); K/V tiles of 64 keys go through shared memory;
// S = Q K^T and O += P V run on mma.sync m16n8k16 (bf16 in, fp32 accumulate);
// the softmax is online in fp32 with exp2.  Query row s (absolute position
// pos_offset + s) sees keys 0 .. pos_offset + s, as attention.py:85-87.
__global__ void __launch_bounds__(128) attn_prefill_kernel(const bf16* __restrict__ q, const bf16* __restrict__ kc,
                                                           const bf16* __restrict__ vc, bf16* __restrict__ out, int H,
                                                           int KVH, int S, int smax, int pos_offset,
                                                           float scale_log2) {
  __shared__ __align__(16) bf16 sK[kBK][kPad];
  __shared__ __align__(16) bf16 sV[kBK][kPad];
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

  for (int k0 = 0; k0 < kmax; k0 += kBK) {
    __syncthreads();  // previous tile fully consumed
    for (int v = threadIdx.x; v < kBK * kHD / 8; v += 128) {
      const int row = v / (kHD / 8), c8 = (v % (kHD / 8)) * 8;
      int4 kv = make_int4(0, 0, 0, 0), vv = make_int4(0, 0, 0, 0);
      if (k0 + row < total) {
        kv = *reinterpret_cast<const int4*>(kp + (int64_t)(k0 + row) * kHD + c8);
        vv = *reinterpret_cast<const int4*>(vp + (int64_t)(k0 + row) * kHD + c8);
      }
      *reinterpret_cast<int4*>(&sK[row][c8]) = kv;
      *reinterpret_cast<int4*>(&sV[row][c8]) = vv;
    }
    __syncthreads();

    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&sK[nt * 8 + g][kk * 16 + 2 * t]);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&sK[nt * 8 + g][kk * 16 + 8 + 2 * t]);
        mma_bf16_16816(s[nt], qa[kk], b0, b1);
      }
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
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
        ldmatrix_x4_trans(vb, &sV[kk * 16 + (mi & 1) * 8 + r][dt * 8 + (mi >> 1) * 8]);
        mma_bf16_16816(o[dt], pa, vb[0], vb[1]);
        mma_bf16_16816(o[dt + 1], pa, vb[2], vb[3]);
      }
    }
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

// One CTA per (batch, KV head) serves the H/KVH query heads that share it, so
// each cached key / value row is read once per step.  Every phase is
// parallel over keys (no serial chain over the context):
//   1. scores: thread t takes keys t, t+256, ...; q (fp32) is broadcast from
//      shared memory; scores go to smem [n_rep][total];
//   2. softmax per head (one warp per head), P rounded to bf16 as the
//      prefill kernel does;
//   3. P@V: warp w takes keys w, w+8, ...; lane l owns dims 2l, 2l+1 of every
//      head; the 8 warps' partial sums are added through shared memory.
__global__ void __launch_bounds__(256) attn_decode_kernel(const bf16* __restrict__ q, const bf16* __restrict__ kc,
                                                          const bf16* __restrict__ vc, bf16* __restrict__ out, int H,
                                                          int KVH, int smax, int total, float scale_log2) {
  extern __shared__ float dsm[];  // sc [n_rep][total], then red [8][n_rep][kHD]
  __shared__ float qs[16][kHD];
  __shared__ float lsum[16];
  const int b = blockIdx.x, kvh = blockIdx.y;
  const int n_rep = H / KVH;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sc = dsm;
  float* red = dsm + n_rep * total;
  for (int i = threadIdx.x; i < n_rep * kHD; i += 256) {
    const int r = i / kHD, d = i % kHD;
    qs[r][d] = __bfloat162float(q[((int64_t)b * H + kvh * n_rep + r) * kHD + d]);
  }
  __syncthreads();
  const bf16* kp = kc + ((int64_t)(b * KVH + kvh) * smax) * kHD;
  const bf16* vp = vc + ((int64_t)(b * KVH + kvh) * smax) * kHD;

  for (int key = threadIdx.x; key < total; key += 256) {
    float acc[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) acc[r] = 0.0f;
    const int4* krow = reinterpret_cast<const int4*>(kp + (int64_t)key * kHD);
#pragma unroll
    for (int c = 0; c < kHD / 8; ++c) {
      const int4 raw = __ldg(krow + c);
      const __nv_bfloat162* kv = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float kx = __low2float(kv[e]), ky = __high2float(kv[e]);
        const int d = c * 8 + 2 * e;
#pragma unroll
        for (int r = 0; r < 16; ++r)
          if (r < n_rep) acc[r] += qs[r][d] * kx + qs[r][d + 1] * ky;
      }
    }
#pragma unroll
    for (int r = 0; r < 16; ++r)
      if (r < n_rep) sc[r * total + key] = acc[r] * scale_log2;
  }
  __syncthreads();
  for (int r = warp; r < n_rep; r += 8) {
    float mx = -INFINITY;
    for (int k = lane; k < total; k += 32) mx = fmaxf(mx, sc[r * total + k]);
#pragma unroll
    for (int o_ = 16; o_ > 0; o_ >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o_));
    float sum = 0.0f;
    for (int k = lane; k < total; k += 32) {
      const float p = ex2_approx(sc[r * total + k] - mx);
      sum += p;
      sc[r * total + k] = __bfloat162float(__float2bfloat16_rn(p));
    }
#pragma unroll
    for (int o_ = 16; o_ > 0; o_ >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o_);
    if (lane == 0) lsum[r] = sum;
  }
  __syncthreads();
  float ax[16], ay[16];
#pragma unroll
  for (int r = 0; r < 16; ++r) ax[r] = ay[r] = 0.0f;
#pragma unroll 4
  for (int k = warp; k < total; k += 8) {
    const __nv_bfloat162 vv = reinterpret_cast<const __nv_bfloat162*>(vp + (int64_t)k * kHD)[lane];
    const float vx = __low2float(vv), vy = __high2float(vv);
#pragma unroll
    for (int r = 0; r < 16; ++r)
      if (r < n_rep) {
        const float p = sc[r * total + k];
        ax[r] += p * vx;
        ay[r] += p * vy;
      }
  }
#pragma unroll
  for (int r = 0; r < 16; ++r)
    if (r < n_rep) {
      red[(warp * n_rep + r) * kHD + 2 * lane] = ax[r];
      red[(warp * n_rep + r) * kHD + 2 * lane + 1] = ay[r];
    }
  __syncthreads();
  for (int i = threadIdx.x; i < n_rep * kHD; i += 256) {
    const int r = i / kHD, d = i % kHD;
    float acc = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) acc += red[(w * n_rep + r) * kHD + d];
    out[((int64_t)b * H + kvh * n_rep + r) * kHD + d] = __float2bfloat16_rn(acc / lsum[r]);
  }
}

// ----------------------------------------------------------------------------- argmax

// Is (v2, i2) a better argmax candidate than (v1, i1)?  Larger value wins,
// ties go to the smaller index, NaN counts as the maximum (torch.argmax);
// an index >= cols marks "no candidate yet".
__device__ __forceinline__ bool better(float v1, int64_t i1, float v2, int64_t i2, int64_t cols) {
  if (i2 >= cols) return false;
  if (i1 >= cols) return true;
  const bool n1 = v1 != v1, n2 = v2 != v2;
  if (n1 || n2) return n1 && n2 ? i2 < i1 : n2;
  return v2 > v1 || (v2 == v1 && i2 < i1);
}

// idx[r] = first index of the maximum of logits[r, :].
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ x, int64_t cols, int64_t ld,
                                                      int64_t* __restrict__ idx) {
  __shared__ float sv[32];
  __shared__ int64_t si[32];
  const float* row = x + (int64_t)blockIdx.x * ld;
  float best = 0.0f;
  int64_t bi = cols;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
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
  embedding_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, (cudaStream_t)stream>>>(
      static_cast<const bf16*>(table), ids, static_cast<bf16*>(out), rows, dim, vocab, bad);
  return check_launch("xb_embedding_bf16", err, errlen);
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
  if (!qkv || !cos_t || !sin_t || !q_out || !k_cache || !v_cache) {
    set_err(err, errlen, "xb_rope_kv_bf16: null pointer");
    return XB_ERR_INVALID;
  }
  const int64_t total = batch * seq * (n_head + 2 * n_kv_head) * (head_dim / 2);
  int64_t grid = (total + 255) / 256;
  if (grid > 148 * 64) grid = 148 * 64;
  rope_kv_kernel<<<(unsigned)grid, 256, 0, (cudaStream_t)stream>>>(
      static_cast<const bf16*>(qkv), cos_t, sin_t, static_cast<bf16*>(q_out), static_cast<bf16*>(k_cache),
      static_cast<bf16*>(v_cache), (int)batch, (int)seq, (int)n_head, (int)n_kv_head, (int)head_dim, (int)max_seq,
      (int)pos_offset);
  return check_launch("xb_rope_kv_bf16", err, errlen);
}

extern "C" int xb_attention_bf16(const void* q, const void* k_cache, const void* v_cache, void* out, int64_t batch,
                                 int64_t seq, int64_t n_head, int64_t n_kv_head, int64_t head_dim, int64_t max_seq,
                                 int64_t pos_offset, float scale, void* stream, char* err, size_t errlen) {
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
    if (n_rep > 16) {
      set_err(err, errlen, "%s: more than 16 query heads per KV head", what);
      return XB_ERR_UNSUPPORTED;
    }
    const size_t smem = ((size_t)n_rep * total + 8 * (size_t)n_rep * kHD) * sizeof(float);
    if (smem > 200 * 1024) {
      set_err(err, errlen, "%s: decode context %d too long for the score buffer", what, total);
      return XB_ERR_UNSUPPORTED;
    }
    static size_t smem_set = 48 * 1024;
    if (smem > smem_set) {
      cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      smem_set = 200 * 1024;
    }
    attn_decode_kernel<<<dim3((unsigned)batch, (unsigned)n_kv_head), 256, smem, s>>>(
        static_cast<const bf16*>(q), static_cast<const bf16*>(k_cache), static_cast<const bf16*>(v_cache),
        static_cast<bf16*>(out), (int)n_head, (int)n_kv_head, (int)max_seq, total, scale_log2);
  } else {
    dim3 grid((unsigned)((seq + kBQ - 1) / kBQ), (unsigned)(batch * n_head));
    attn_prefill_kernel<<<grid, 128, 0, s>>>(static_cast<const bf16*>(q), static_cast<const bf16*>(k_cache),
                                             static_cast<const bf16*>(v_cache), static_cast<bf16*>(out),
                                             (int)n_head, (int)n_kv_head, (int)seq, (int)max_seq, (int)pos_offset,
                                             scale_log2);
  }
  return check_launch(what, err, errlen);
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
  argmax_kernel<<<(unsigned)rows, 1024, 0, (cudaStream_t)stream>>>(x, cols, ld, idx);
  return check_launch("xb_argmax_f32", err, errlen);
}
