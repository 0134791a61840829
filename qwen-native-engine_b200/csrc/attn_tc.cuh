// Paged-KV attention decode step on the tensor cores (mma.sync m16n8k16, f16 in, f32
// accumulate); same work item, prologue and split merge as AttnItem (attn_dev.cuh), which the
// fused layer kernels keep. Per item = (context split, KV head, sequence), per 64-token
// sub-block:
//   S[token][head] = K q      A = K tile [16 tokens][16 dims] (ldmatrix from shared memory),
//                             B = q of the 4 query heads (columns 4..7 zero), q as hi + lo f16
//                             halves, so the product keeps the f32 query;
//   online softmax over the sub-block per head (as AttnItem);
//   O[dim][head] += V^T P     A = V^T tile (ldmatrix.trans of V rows), B = P as hi + lo f16.
// Warp w computes the scores of tokens 16 (w % 4) .. +15 over dims 128 (w / 4) .. +127 (the two
// halves are summed in the softmax pass), and owns output dims 32 w .. 32 w + 31 of the PV
// product, so no cross-warp reduction of the accumulator is needed.
//
// K and V rows are staged in shared memory with their 16-byte chunks permuted (chunk c of row r
// at c ^ (r % 8)), which makes every ldmatrix phase touch 8 different bank groups. K of the next
// sub-block is staged while this one's softmax and PV run, V of the next while its scores run.
#pragma once

#include "attn_dev.cuh"

namespace qne {
namespace dev {

// C = the MMA columns in use: the 4 query heads of the KV head for each of the item's query rows
// (C = 4: one row; C = 8: two rows, the prompt path).
template <int C>
struct AttnTcSharedT {
  __align__(128) uint4 kst[kSub][kHeadDim / 8];  // 64 tokens x 32 chunks of 8 f16, permuted
  __align__(128) uint4 vst[kSub][kHeadDim / 8];
  __align__(16) float q_s[C][kHeadDim];
  __align__(16) float kc_s[kHeadDim];  // the current token's key and value (f16-rounded)
  __align__(16) float vc_s[kHeadDim];
  // Rows padded by 8 floats so the columns' rows start in different banks (the PV fragment loads
  // read the same token offset of all columns at once).
  float spart[2][C][kSub + 8];  // scores of the two dim halves
  float sc[C][kSub + 8];        // probabilities of the sub-block
  float red[8][kQPerKv];
  float redk[8];
  float blk_scale[C];
  float run_m[C], run_l[C];
  uint32_t flag;
  // After the last sub-block: the output accumulator [C columns][256 dims], in the K area.
  __device__ __forceinline__ float* o_s() { return reinterpret_cast<float*>(&kst[0][0]); }
  static_assert(sizeof(kst) >= C * kHeadDim * sizeof(float), "o_s aliases the K staging area");
  static_assert(C == 4 || C == 8, "one or two query rows per item");
};
using AttnTcShared = AttnTcSharedT<4>;

__device__ __forceinline__ int swz(int row, int chunk) { return chunk ^ (row & 7); }

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  return (uint32_t)__half_as_ushort(__float2half_rn(a)) | ((uint32_t)__half_as_ushort(__float2half_rn(b)) << 16);
}
// hi = f16(x), lo = f16(x - hi) for two values, packed as f16x2 (low half = first value).
__device__ __forceinline__ void hilo2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __half ah = __float2half_rn(a), bh = __float2half_rn(b);
  hi = (uint32_t)__half_as_ushort(ah) | ((uint32_t)__half_as_ushort(bh) << 16);
  lo = pack_h2(a - __half2float(ah), b - __half2float(bh));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_attn(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// G = query rows per item (1: decode; 2: the prompt path, whose rows are consecutive positions
// of one sequence reading one cache, kv_appended and page_table_stride 0).
template <int G>
struct AttnTcItemT {
  static constexpr int kCols = 4 * G;
  using Shared = AttnTcSharedT<kCols>;
  int split, kvh, b, len, nsplit, l0, l1;
  uint32_t pos;
  bool valid, owner;
  const uint32_t* pt;
  uint32_t pos_r[G];   // position of each query row (pos = the largest)
  bool rowok[G];       // row inside the batch
  float4 cst[G];       // attn_consts at each row's position

  // Stages K (kind 0) or V (kind 1) of the 64 tokens from sb and commits them as one cp.async
  // group (an empty group past the split's end). Thread t copies chunk t % 32 of rows t / 32 +
  // 8 i. Rows outside [l0, l1) and rows of an out-of-range page are zero-filled; the row of the
  // token this item appends is left to patch_current(). The sub-block's four page ids are read
  // together (row t / 32 + 8 i lies in page i / 2; sb <= 4032, so the ids stay inside the
  // 256-entry table), one round trip before the copies instead of one per row.
  __device__ __forceinline__ void stage(const KernelArgs& ka, Shared& sh, int sb, int kind) const {
    uint32_t pg[4];
    if (sb < l1) load_pages(sb, pg);
    stage_pages(ka, sh, sb, kind, pg);
  }
  __device__ __forceinline__ void load_pages(int sb, uint32_t (&pg)[4]) const {
    static_assert(kSub == 4 * kPageTokens, "a sub-block spans four pages");
#pragma unroll
    for (int p = 0; p < 4; ++p) pg[p] = pt[sb / kPageTokens + p];
  }
  __device__ __forceinline__ void stage_pages(const KernelArgs& ka, Shared& sh, int sb, int kind,
                                              const uint32_t (&pg)[4]) const {
    const int t = threadIdx.x, c = t & 31;
    if (sb < l1) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = (t >> 5) + 8 * i, l = sb + r;
        if (owner && l == (int)pos) continue;
        uint4* d = kind == 0 ? &sh.kst[r][swz(r, c)] : &sh.vst[r][swz(r, c)];
        const uint32_t page = l < l1 ? pg[i >> 1] : 0xFFFFFFFFu;
        if (page < ka.pool_pages) cp_async16_attn(d, kv_row(ka.a.kv, page, kind, kvh, l % kPageTokens) + c * 8);
        else *d = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }

  // Writes the appended token's f16 key and value rows into the staging area (sub-block sb).
  __device__ __forceinline__ void patch_current(Shared& sh, int sb) const {
    const int t = threadIdx.x;
    if (!owner || (int)pos < sb || (int)pos >= sb + kSub || t >= 64) return;
    const int r = (int)pos - sb, c = t & 31;
    const float* src = (t < 32 ? sh.kc_s : sh.vc_s) + c * 8;
    uint4 v;
    v.x = pack_h2(src[0], src[1]);
    v.y = pack_h2(src[2], src[3]);
    v.z = pack_h2(src[4], src[5]);
    v.w = pack_h2(src[6], src[7]);
    (t < 32 ? sh.kst : sh.vst)[r][swz(r, c)] = v;
  }

  __device__ __forceinline__ void prefetch(const KernelArgs& ka, Shared& sh, int item) {
    const AttnArgs& a = ka.a;
    split = item % ka.max_splits;
    kvh = (item / ka.max_splits) % kKvHeads;
    b = (item / (ka.max_splits * kKvHeads)) * G;
    // The first sub-block's page ids do not depend on the positions: requested with them.
    pt = a.page_table + (size_t)b * a.page_table_stride;
    uint32_t pg[4];
    load_pages(split * ka.split, pg);
    pos = 0;
#pragma unroll
    for (int r = 0; r < G; ++r) {
      rowok[r] = b + r < a.batch;
      uint32_t p = rowok[r] ? a.pos[(size_t)(b + r) * a.pos_stride] : 0u;
      if (p >= (uint32_t)kMaxContext) {
        if (a.flags && threadIdx.x == 0 && split == 0 && kvh == 0)
          atomicOr(a.flags + (size_t)(b + r) * a.flags_stride, kFlagPosClamped);
        p = kMaxContext - 1;
      }
      pos_r[r] = p;
      if (rowok[r] && p > pos) pos = p;
    }
    len = (int)pos + 1;
    nsplit = (len + ka.split - 1) / ka.split;
    valid = split < nsplit;
    if (!valid) return;
    l0 = split * ka.split;
    l1 = min(l0 + ka.split, len);
    owner = G == 1 && !a.kv_appended && (int)pos >= l0 && (int)pos < l1;
#pragma unroll
    for (int r = 0; r < G; ++r) cst[r] = attn_consts(a, pos_r[r]);
    stage_pages(ka, sh, l0, 0, pg);
    stage_pages(ka, sh, l0, 1, pg);
  }

  __device__ __forceinline__ void run(const KernelArgs& ka, Shared& sh) {
    const AttnArgs& a = ka.a;
    if (!valid) return;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int g = lane >> 2, tq = lane & 3;
#pragma unroll 1
    for (int r = 0; r < G; ++r) {
      if (rowok[r]) {
        attn_prologue(ka, sh, b + r, kvh, pos_r[r], owner && r == 0, pt, cst[r], 4 * r);
      } else {  // a row past the batch: zero query, an empty softmax, never stored
#pragma unroll
        for (int hh = 0; hh < kQPerKv; ++hh) sh.q_s[4 * r + hh][t] = 0.f;
        if (t < kQPerKv) {
          sh.run_m[4 * r + t] = -INFINITY;
          sh.run_l[4 * r + t] = 0.f;
        }
        __syncthreads();
      }
    }

    // B fragments of q (head g, zero for g >= 4) for this warp's dim half: 8 k-steps, hi and lo.
    const int dh = warp >> 2, tt = warp & 3;
    uint32_t qh[8][2], ql[8][2];
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int d = dh * 128 + kk * 16 + 2 * tq;
      float q0 = 0.f, q1 = 0.f, q2 = 0.f, q3 = 0.f;
      if (g < kCols) {
        q0 = sh.q_s[g][d];
        q1 = sh.q_s[g][d + 1];
        q2 = sh.q_s[g][d + 8];
        q3 = sh.q_s[g][d + 9];
      }
      hilo2(q0, q1, qh[kk][0], ql[kk][0]);
      hilo2(q2, q3, qh[kk][1], ql[kk][1]);
    }
    float acc[2][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[m][e] = 0.f;
    const uint32_t kbase = (uint32_t)__cvta_generic_to_shared(&sh.kst[0][0]);
    const uint32_t vbase = (uint32_t)__cvta_generic_to_shared(&sh.vst[0][0]);
    const int mi = lane >> 3, mr = lane & 7;  // ldmatrix: matrix index and row of this lane

    // Cp.async groups are committed K0 V0 K1 V1 ...; at each wait the one newer group may stay
    // in flight, and a barrier makes every thread's chunks visible to the ldmatrix readers.
#pragma unroll 1
    for (int sb = l0; sb < l1; sb += kSub) {
      patch_current(sh, sb);
      asm volatile("cp.async.wait_group 1;" ::: "memory");  // K(sb)
      __syncthreads();
      {
        float s[4] = {0.f, 0.f, 0.f, 0.f};
        const int row = tt * 16 + mr + 8 * (mi & 1);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const int chunk = dh * 16 + kk * 2 + (mi >> 1);
          uint32_t a0, a1, a2, a3;
          ldsm_x4(kbase + (uint32_t)((row * 32 + swz(row, chunk)) * 16), a0, a1, a2, a3);
          mma_attn(s, a0, a1, a2, a3, qh[kk][0], qh[kk][1]);
          mma_attn(s, a0, a1, a2, a3, ql[kk][0], ql[kk][1]);
        }
        if (2 * tq < kCols) {
          sh.spart[dh][2 * tq][tt * 16 + g] = s[0];
          sh.spart[dh][2 * tq + 1][tt * 16 + g] = s[1];
          sh.spart[dh][2 * tq][tt * 16 + g + 8] = s[2];
          sh.spart[dh][2 * tq + 1][tt * 16 + g + 8] = s[3];
        }
      }
      __syncthreads();  // K(sb) is read, the score halves are visible
      stage(ka, sh, sb + kSub, 0);
      {
        // Online softmax per column: thread (hh = t / 64, j = t % 64) takes token j of columns
        // hh + 4 r (query head hh of each row r; a row's tokens end at its own position).
        const int hh = t >> 6, j = t & 63;
        float sval[G];
#pragma unroll
        for (int r = 0; r < G; ++r) {
          const int c = hh + 4 * r;
          const int lim = G == 1 ? l1 : min(l1, (int)pos_r[r] + 1);
          sval[r] = (rowok[r] && sb + j < lim) ? sh.spart[0][c][j] + sh.spart[1][c][j] : -INFINITY;
          const float m = warp_max(sval[r]);
          if (lane == 0) sh.red[warp][2 * r] = m;
        }
        __syncthreads();
        if (j == 0) {
#pragma unroll
          for (int r = 0; r < G; ++r) {
            const int c = hh + 4 * r;
            const float mb = fmaxf(sh.red[2 * hh][2 * r], sh.red[2 * hh + 1][2 * r]);
            const float mnew = fmaxf(sh.run_m[c], mb);
            sh.blk_scale[c] = (sh.run_m[c] == -INFINITY) ? 0.f : expf(sh.run_m[c] - mnew);
            sh.run_m[c] = mnew;
          }
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < G; ++r) {
          const int c = hh + 4 * r;
          const float p = (sval[r] == -INFINITY) ? 0.f : expf(sval[r] - sh.run_m[c]);
          sh.sc[c][j] = p;
          const float ps = warp_sum(p);
          if (lane == 0) sh.red[warp][2 * r + 1] = ps;
        }
        asm volatile("cp.async.wait_group 1;" ::: "memory");  // V(sb)
        __syncthreads();
        if (j == 0) {
#pragma unroll
          for (int r = 0; r < G; ++r) {
            const int c = hh + 4 * r;
            sh.run_l[c] = sh.run_l[c] * sh.blk_scale[c] + sh.red[2 * hh][2 * r + 1] + sh.red[2 * hh + 1][2 * r + 1];
          }
        }
      }
      {
        // O[dim][head] (dims 32 warp .. +31) = blk_scale * O + V^T P.
        float f0 = 0.f, f1 = 0.f;
        if (2 * tq < kCols) {
          f0 = sh.blk_scale[2 * tq];
          f1 = sh.blk_scale[2 * tq + 1];
        }
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          acc[m][0] *= f0;
          acc[m][1] *= f1;
          acc[m][2] *= f0;
          acc[m][3] *= f1;
        }
#pragma unroll
        for (int kt = 0; kt < kSub / 16; ++kt) {
          float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
          if (g < kCols) {
            p0 = sh.sc[g][kt * 16 + 2 * tq];
            p1 = sh.sc[g][kt * 16 + 2 * tq + 1];
            p2 = sh.sc[g][kt * 16 + 2 * tq + 8];
            p3 = sh.sc[g][kt * 16 + 2 * tq + 9];
          }
          uint32_t ph0, pl0, ph1, pl1;
          hilo2(p0, p1, ph0, pl0);
          hilo2(p2, p3, ph1, pl1);
          const int row = kt * 16 + mr + 8 * (mi >> 1);  // V row (token) this lane addresses
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            const int chunk = warp * 4 + m * 2 + (mi & 1);
            uint32_t a0, a1, a2, a3;
            ldsm_x4_t(vbase + (uint32_t)((row * 32 + swz(row, chunk)) * 16), a0, a1, a2, a3);
            mma_attn(acc[m], a0, a1, a2, a3, ph0, ph1);
            mma_attn(acc[m], a0, a1, a2, a3, pl0, pl1);
          }
        }
      }
      __syncthreads();  // V(sb) and the probabilities are read
      stage(ka, sh, sb + kSub, 1);
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");  // (only empty groups remain)
    __syncthreads();  // o_s reuses the K area
    float* os = sh.o_s();
    if (2 * tq < kCols) {
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const int d = warp * 32 + m * 16 + g;
        os[(2 * tq) * kHeadDim + d] = acc[m][0];
        os[(2 * tq + 1) * kHeadDim + d] = acc[m][1];
        os[(2 * tq) * kHeadDim + d + 8] = acc[m][2];
        os[(2 * tq + 1) * kHeadDim + d + 8] = acc[m][3];
      }
    }
    __syncthreads();
#pragma unroll 1
    for (int r = 0; r < G; ++r) {
      const int nsplit_r = ((int)pos_r[r] + ka.split) / ka.split;  // splits of row r: ceil((pos + 1) / split)
      if (!rowok[r] || split >= nsplit_r) continue;  // uniform across the CTA
      const float4 o = *reinterpret_cast<const float4*>(os + (4 * r + (t >> 6)) * kHeadDim + (t & 63) * 4);
      attn_merge_store(a, sh, b + r, kvh, split, nsplit_r, o, 4 * r, ka.spread != 0);
    }
  }
};
using AttnTcItem = AttnTcItemT<1>;

}  // namespace dev
}  // namespace qne
