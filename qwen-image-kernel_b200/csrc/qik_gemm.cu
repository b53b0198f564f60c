// qik_gemm.cu -- FP8 (e4m3 x e4m3 -> fp32) GEMM on the sm_100a tensor core.
//
// C[M,N] = epilogue(A[M,K] . B[N,K]^T): the W8A8 per-tensor linear of
// FP8Linear.forward (qwen_image_kernel/fp8.py:78-90), whose reference computes it
// with torch._scaled_mm.  Design:
//   * persistent CTAs, output tiles visited round-robin, in one of two modes:
//     - CTA pairs (clusters of 2, the default from M = 512): 256 x 256 tiles computed
//       by tcgen05.mma.cta_group::2 -- each CTA loads 128 rows of A and 128 rows of B
//       per stage, so a CTA moves 32 KB instead of 48 KB per 128-deep K step for the
//       same 128 x 256 share of the output, with 6 pipeline stages;
//     - single CTAs with 128 x BN tiles (BN = 256, 128 or 64) for skinny M, and for at
//       most 16 rows the operands swapped (BN = 16: 128 weight rows x 16 activation
//       rows per tile, stored transposed by the epilogue);
//   * warp 0: TMA producer -- 128-byte swizzle, no cluster multicast (each CTA loads
//     its own tiles; in a pair both CTAs' loads complete on the leader's barrier);
//   * warp 1: one thread (of the leader CTA in a pair) issues tcgen05.mma.kind::f8f6f4
//     (K = 32 per instruction) into a double-buffered fp32 accumulator in tensor
//     memory and releases smem stages / accumulators with tcgen05.commit (multicast
//     to both CTAs of a pair);
//   * warps 2-9: epilogue -- tcgen05.ld of the CTA's own accumulator rows, scale by
//     sa*sb, optional bias and GELU-tanh, bf16/fp32 via swizzled staging and TMA
//     stores, optional amax of the bf16 output for the next dynamic quantization;
//     or (QIK_EPI_SWIGLU) silu(gate) * up of a CTA-pair tile whose leader loaded 128
//     gate rows of the fused up-projection weight and whose peer the matching 128 up
//     rows, so each tile's TMEM holds both operands of 128 output columns;
//     or (QIK_EPI_RMS_ROPE, the fused QKV linear) the per-head RMSNorm + RoPE of the q
//     and k heads, one head per warp: the squares of the bf16 outputs summed in the
//     RMSNorm + RoPE kernel's order, then the accumulator read again and normalised,
//     rotated and stored (bit-identical to GEMM -> qik_rms_norm_rope);
//     or (QIK_EPI_SCATTER) fp32 rows stored from the staging buffer straight into the
//     owner rank's receive slot in peer memory, each finished tile counted there.
// The epilogue of tile i overlaps the MMAs of tile i+1.
#include <string.h>

#include <mutex>

#include "qik_device.cuh"
#include "qik_host.h"

namespace qik {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 128;  // e4m3 elements (= bytes) of K per pipeline stage
constexpr int kGemmEpiWarps = 8;                  // two per TMEM lane quarter
constexpr int kGemmThreads = 64 + 32 * kGemmEpiWarps;

struct GemmParams {
  int M, N, K;
  const float* scale_a;
  const float* scale_b;
  const __nv_bfloat16* bias;
  void* C;
  int64_t ldc;
  int out_f32;
  int epilogue;
  uint32_t* amax_out;
  int* status;
  // QIK_EPI_SCATTER (row-parallel partial products reduced over peer memory): row r
  // of the fp32 result goes to scat_dst[r / scat_rows] + (r % scat_rows) * N, and each
  // CTA counts every finished tile at scat_cnt[owner] (system-scope atomic).
  float* scat_dst[QIK_TP_MAX_WORLD];
  uint32_t* scat_cnt[QIK_TP_MAX_WORLD];
  int scat_rows;
  int group_m;  // raster: row tiles per group (1 = row-major), see tile_coords
  int keep_out_l2;  // bf16 output stored with an L2 evict-last policy (its consumer follows at once)
  // QIK_EPI_RMS_ROPE (the fused QKV linear): columns [0, rms_cols) are the q heads then
  // the k heads, 128 columns each, normalised with rms_w[0] (the first rms_cols / 2
  // columns) or rms_w[1] and rotated by rope_cos / rope_sin [rope_seq, 64] at position
  // row % rope_seq; the columns after them (v) as QIK_EPI_SCALE
  const float* rms_w[2];
  const float* rope_cos;
  const float* rope_sin;
  int rope_seq;
  int rms_cols;
  float rms_eps;
  // QIK_EPI_GATE_RES (the DiT block's gated residual): C = x + bf16(T[t] * f) with f the
  // bf16 output, x = res_x [M, N] (row pitch res_ld), T the bf16(tanh(gate)) table (row
  // pitch gate_ld) and t = b + (gate_mask && !gate_mask[s] ? gate_batch : 0) for row
  // b * gate_seq + s
  const uint16_t* res_x;
  int64_t res_ld;
  const uint16_t* gate_tab;
  int64_t gate_ld;
  const uint8_t* gate_mask;
  int gate_seq;
  int gate_batch;
};

// Output tile `tile` of the raster: groups of group_m row tiles, each group walked
// column tile by column tile with its row tiles fastest.  Consecutive tiles (the CTAs
// of one wave) then share a few row bands of A and a few column bands of B instead of
// one row band and all of B, so a B larger than what L2 keeps between waves is read
// from HBM once per group rather than once per wave.  group_m = 1 is row-major.
__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int group_m, int& mb, int& nb) {
  const int per_group = group_m * num_n;
  const int g = tile / per_group;
  const int first = g * group_m;
  const int gm = min(num_m - first, group_m);
  const int r = tile - g * per_group;
  mb = first + r % gm;
  nb = r / gm;
}

// TWO_SM: the CTA is half of a 2-CTA cluster computing 256 x BN tiles with
// tcgen05.mma.cta_group::2 -- it loads 128 rows of A and BN / 2 rows of B per stage.
template <int BN, int STAGES, bool TWO_SM = false>
struct GemmLayout {
  static constexpr int kABytes = kGemmBM * kGemmBK;
  static constexpr int kBBytes = (TWO_SM ? BN / 2 : BN) * kGemmBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStageOutOffset = STAGES * kStageBytes;  // 8 warps x 2 buffers x 2 KB
  static constexpr int kOutBufBytes = 2048;                      // 32 rows x 64 bytes
  // the transposed tiny-M form (BN = 16) stores straight from registers: no staging
  static constexpr int kBarOffset = kStageOutOffset + (BN == 16 ? 0 : kGemmEpiWarps * 2 * kOutBufBytes);
  static constexpr int kBarBytes = (2 * STAGES + 4) * 8 + 16;
  static constexpr int kSmemBytes = kBarOffset + kBarBytes + 1024;  // + alignment slack
  // two accumulators of BN columns each (BN a power of two, as the TMEM allocation is)
  static constexpr int kAccStride = BN;
  static constexpr int kTmemCols = 2 * BN;
};

// GELU, tanh form: 0.5 x (1 + tanh(u)), u = sqrt(2/pi) (x + 0.044715 x^3), evaluated
// through the identity 0.5 (1 + tanh(u)) = 1 / (1 + e^(-2u)) with the MUFU exp2 and
// reciprocal (PTX ex2.approx / rcp.approx, both within ~2 ulp of fp32): relative
// accuracy stays at fp32 level on both tails, far below the bf16 rounding that follows.
__device__ __forceinline__ float gelu_tanh_f32(float x) {
  const float k0 = 0.7978845608028654f;   // sqrt(2/pi)
  const float k1 = 0.044715f;
  const float u = k0 * fmaf(k1 * x, x * x, x);
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(u * -2.8853900817779268f));  // e^(-2u) = 2^(-2u log2 e)
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
  return x * r;
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// v[j] += bias[j] for j < ncols (16 or 32), the bias row 16-byte aligned
__device__ __forceinline__ void add_bias32(float (&v)[32], const __nv_bfloat16* bias, int ncols = 32) {
  const uint4* bp = reinterpret_cast<const uint4*>(bias);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 bb = (q * 8 < ncols) ? __ldg(bp + q) : make_uint4(0u, 0u, 0u, 0u);
    const uint32_t bw[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      v[q * 8 + 2 * t] += __uint_as_float(bw[t] << 16);
      v[q * 8 + 2 * t + 1] += __uint_as_float(bw[t] & 0xFFFF0000u);
    }
  }
}

// Epilogue kinds compiled into separate kernels, so the plain path carries none of the
// fused epilogues' code: plain (QIK_EPI_SCALE / GELU_TANH / SCATTER), SwiGLU, RMSNorm +
// RoPE (CTA pairs only) and gated residual.
constexpr int kEkPlain = 0, kEkSwiglu = 1, kEkRms = 2, kEkGate = 3;

template <int BN, int STAGES, bool TWO_SM, int EK>
__global__ void __launch_bounds__(kGemmThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
  using Lay = GemmLayout<BN, STAGES, TWO_SM>;
  constexpr int kTileM = TWO_SM ? 2 * kGemmBM : kGemmBM;  // output rows per tile
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Lay::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Lay::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = TWO_SM ? cluster_ctarank() : 0u;  // 0 = leader (issues the MMAs)
  // tile index, and the stride over tiles: one per CTA, or one per CTA pair
  const int tile0 = TWO_SM ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int tile_step = TWO_SM ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      // the leader's accumulator is free once the epilogue warps of both CTAs drained it
      mbar_init(&tempty[a], TWO_SM ? 2 * kGemmEpiWarps : kGemmEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    if constexpr (TWO_SM) {
      tmem_alloc_cg2(tmem_slot, Lay::kTmemCols);
      tmem_relinquish_cg2();
    } else {
      tmem_alloc(tmem_slot, Lay::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (TWO_SM) cluster_sync();  // both CTAs' barriers exist before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the set-up above overlaps the predecessor's tail; operands are read below
  pdl_wait();

  const int num_m = (p.M + kTileM - 1) / kTileM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_k = (p.K + kGemmBK - 1) / kGemmBK;
  const int tiles = num_m * num_n;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      // TWO_SM: both CTAs' loads complete on the leader's full barrier, which alone
      // expects the bytes of the pair
      const uint32_t full_leader = TWO_SM ? mapa_shared(full, 0) : 0u;
      // QIK_EPI_SWIGLU: the leader loads gate rows nb * 128 + [0, 128), the peer the up
      // rows N / 2 + nb * 128 + [0, 128), so tile columns 0-127 are gate outputs and
      // 128-255 the matching up outputs
      constexpr bool swiglu = TWO_SM && EK == kEkSwiglu;
      for (int tile = tile0; tile < tiles; tile += tile_step) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, p.group_m, mb, nb);
        const int brow = swiglu ? (rank ? p.N / 2 : 0) + nb * (BN / 2) : nb * BN + static_cast<int>(rank) * (BN / 2);
        for (int kb = 0; kb < num_k; ++kb) {
          if constexpr (TWO_SM) {
            if (!mbar_wait_cluster(&empty[stage], phase ^ 1u, abort_flag, p.status)) goto producer_done;
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * Lay::kStageBytes);
            const uint32_t bar = full_leader + static_cast<uint32_t>(stage) * 8u;
            tma_load_2d_cg2(sA + stage * Lay::kABytes, &tmA, kb * kGemmBK,
                            mb * kTileM + static_cast<int>(rank) * kGemmBM, bar);
            tma_load_2d_cg2(sB + stage * Lay::kBBytes, &tmB, kb * kGemmBK, brow, bar);
          } else {
            if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status)) goto producer_done;
            mbar_arrive_expect_tx(&full[stage], Lay::kStageBytes);
            tma_load_2d(sA + stage * Lay::kABytes, &tmA, kb * kGemmBK, mb * kGemmBM, &full[stage]);
            tma_load_2d(sB + stage * Lay::kBBytes, &tmB, kb * kGemmBK, nb * BN, &full[stage]);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:;
    }
    pdl_trigger();
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_f32acc(0, 0, 0, 0, kTileM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = tile0; tile < tiles; tile += tile_step, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        const bool got = TWO_SM ? mbar_wait_cluster(&tempty[acc], acc_phase ^ 1u, abort_flag, p.status)
                                : mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, p.status);
        if (!got) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * Lay::kAccStride);
        bool ok = true;
        for (int kb = 0; kb < num_k; ++kb) {
          const bool ready = TWO_SM ? mbar_wait_cluster(&full[stage], phase, abort_flag, p.status)
                                    : mbar_wait(&full[stage], phase, abort_flag, p.status);
          if (!ready) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * Lay::kABytes);
          const uint32_t b_addr = smem_u32(sB + stage * Lay::kBBytes);
#pragma unroll
          for (int k = 0; k < kGemmBK / 32; ++k) {
            const uint64_t ad = sdesc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(b_addr + k * 32, 16, 1024);
            if constexpr (TWO_SM)
              umma_f8f6f4_ss_cg2(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
            else
              umma_f8f6f4_ss(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          if constexpr (TWO_SM)
            umma_commit_cg2(&empty[stage], 0x3);  // the stage of both CTAs is free
          else
            umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (TWO_SM)
          umma_commit_cg2(&tfull[acc], 0x3);  // both CTAs' halves of the accumulator are ready
        else
          umma_commit(&tfull[acc]);
      }
    }
    pdl_trigger();
  } else {
    // epilogue warps 2..9: TMEM lane quarter = warp % 4, two warps per quarter take
    // alternate 32-column chunks.  Each warp turns its 32 accumulator rows into
    // output blocks: registers -> swizzled staging buffer (two per warp, alternating)
    // -> one TMA tensor store per block, which writes whole rows coalesced and clips
    // rows >= M / columns >= N.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const float s = __ldg(p.scale_a) * __ldg(p.scale_b);
    uint8_t* stage_out = smem + Lay::kStageOutOffset + (warp - 2) * 2 * Lay::kOutBufBytes;
    uint32_t amax_local = 0;
    int local = 0;
    int buf = 0;
    for (int tile = tile0; tile < tiles; tile += tile_step, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      const bool got = TWO_SM ? mbar_wait_cluster(&tfull[acc], acc_phase, abort_flag, p.status)
                              : mbar_wait(&tfull[acc], acc_phase, abort_flag, p.status);
      if (!got) break;
      tc_fence_after();
      if (tile + tile_step >= tiles) pdl_trigger();  // last tile of this CTA
      int mb, nb;
      tile_coords(tile, num_m, num_n, p.group_m, mb, nb);
      const int row0 = mb * kTileM + static_cast<int>(rank) * kGemmBM + quarter * 32;
      const bool row_ok = row0 + lane < p.M;

      if constexpr (BN == 16) {
        // transposed tiny-M form: kernel row r = output column (a weight row), kernel
        // column c = output row (an activation row); one warp per lane quarter stores
        // its 32 output columns of each of the 16 (valid) output rows, 64 contiguous
        // bytes per row and store
        if (half == 0) {
          uint32_t r[16];
          tmem_ld16(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                        static_cast<uint32_t>(acc * Lay::kAccStride),
                    r);
          const int n = row0 + lane;
          if (row_ok) {
            const float bn = p.bias ? __bfloat162float(p.bias[n]) : 0.0f;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int m = nb * 16 + j;
              if (m >= p.N) break;
              float v = __uint_as_float(r[j]) * s + bn;
              if (p.out_f32) {
                static_cast<float*>(p.C)[static_cast<int64_t>(m) * p.ldc + n] = v;
              } else {
                if (p.epilogue == QIK_EPI_GELU_TANH) v = gelu_tanh_f32(__bfloat162float(__float2bfloat16_rn(v)));
                const __nv_bfloat16 o = __float2bfloat16_rn(v);
                static_cast<__nv_bfloat16*>(p.C)[static_cast<int64_t>(m) * p.ldc + n] = o;
                amax_local = max(amax_local, static_cast<uint32_t>(__bfloat16_as_ushort(o) & 0x7FFFu));
              }
            }
          }
        }
      }
      // 32 rows x 32 bf16 output columns from registers: swizzled staging buffer -> one TMA store
      auto store_bf16 = [&](const uint32_t (&w)[16], int col0) {
        // the staging buffer is free once at most one store (the other buffer's) reads smem
        if (lane == 0) bulk_wait_read_1();
        __syncwarp();
        uint8_t* sb = stage_out + buf * Lay::kOutBufBytes;
        // 64-byte rows, 64-byte swizzle: 16-byte chunk q of row l at chunk q ^ ((l >> 1) & 3)
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(sb + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)) =
              make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && row0 < p.M) {
          if (p.keep_out_l2)
            tma_store_2d_hint(&tmC, col0, row0, sb, l2_evict_last_policy());
          else
            tma_store_2d(&tmC, col0, row0, sb);
          bulk_commit_group();
        }
        buf ^= 1;
      };
      int chunks = BN / 32;
      if constexpr (TWO_SM && BN == 256 && EK == kEkRms) {
        if (nb * 256 < p.rms_cols) {
          // a q or k tile: warp half h takes head h (tile columns 128 h + [0, 128)) whole,
          // so each thread holds its row of the head; pass 1 sums the squares of the bf16
          // outputs in groups of 8 as the RMSNorm + RoPE kernel's lanes do, pass 2 reloads
          // the accumulator, normalises, rotates and stores
          chunks = 0;
          const int hc0 = nb * 256 + half * 128;
          const float* wv = p.rms_w[hc0 >= (p.rms_cols >> 1) ? 1 : 0];
          const uint32_t ta = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                              static_cast<uint32_t>(acc * Lay::kAccStride + half * 128);
          const int srow = (row0 + lane) % p.rope_seq;
          const float4* cs_row = reinterpret_cast<const float4*>(p.rope_cos + static_cast<int64_t>(srow) * 64);
          const float4* sn_row = reinterpret_cast<const float4*>(p.rope_sin + static_cast<int64_t>(srow) * 64);
          // each chunk's 16 cos / sin pairs of this row are loaded one chunk ahead (the
          // first before pass 1), so their L2 latency overlaps the previous chunk's work
          float4 c_nx[4], s_nx[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            c_nx[q] = __ldg(cs_row + q);
            s_nx[q] = __ldg(sn_row + q);
          }
          auto chunk_words = [&](int j, uint32_t (&w)[16]) {
            uint32_t r[32];
            tmem_ld32(ta + static_cast<uint32_t>(j * 32), r);
            float v[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(r[e]) * s;
            if (p.bias) add_bias32(v, p.bias + hc0 + j * 32);
#pragma unroll
            for (int e = 0; e < 16; ++e) w[e] = pack_bf16x2(v[2 * e], v[2 * e + 1]);
          };
          float part[16];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t w[16];
            chunk_words(j, w);
#pragma unroll
            for (int gi = 0; gi < 4; ++gi)
              part[4 * j + gi] = rms_ss8(w[4 * gi], w[4 * gi + 1], w[4 * gi + 2], w[4 * gi + 3]);
          }
          const float rrms = rms_rstd(rms_ss_tree16(part), 128, p.rms_eps);
          const uint64_t rr2 = f2_pack(rrms, rrms);
#pragma unroll 1
          for (int j = 0; j < 4; ++j) {
            float4 c_cur[4], s_cur[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              c_cur[q] = c_nx[q];
              s_cur[q] = s_nx[q];
            }
            if (j < 3) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                c_nx[q] = __ldg(cs_row + (j + 1) * 4 + q);
                s_nx[q] = __ldg(sn_row + (j + 1) * 4 + q);
              }
            }
            uint32_t w[16];
            chunk_words(j, w);
            const float4* wp = reinterpret_cast<const float4*>(wv + j * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float4 wa = __ldg(wp + 2 * q), wb = __ldg(wp + 2 * q + 1);
              const float4 c4 = c_cur[q], s4 = s_cur[q];
              w[4 * q] = rms_rope_pair(w[4 * q], rr2, f2_pack(wa.x, wa.y), f2_pack(c4.x, s4.x), f2_pack(-s4.x, c4.x));
              w[4 * q + 1] =
                  rms_rope_pair(w[4 * q + 1], rr2, f2_pack(wa.z, wa.w), f2_pack(c4.y, s4.y), f2_pack(-s4.y, c4.y));
              w[4 * q + 2] =
                  rms_rope_pair(w[4 * q + 2], rr2, f2_pack(wb.x, wb.y), f2_pack(c4.z, s4.z), f2_pack(-s4.z, c4.z));
              w[4 * q + 3] =
                  rms_rope_pair(w[4 * q + 3], rr2, f2_pack(wb.z, wb.w), f2_pack(c4.w, s4.w), f2_pack(-s4.w, c4.w));
            }
            store_bf16(w, hc0 + j * 32);
          }
        }
      }
      if constexpr (TWO_SM && BN == 256 && EK == kEkSwiglu) {
        {
          // tile columns c * 32 + [0, 32) (gate) and 128 + c * 32 + [0, 32) (up) give output
          // columns nb * 128 + c * 32 + [0, 32); N % 256 == 0, so every chunk is whole
          chunks = 0;
          const int h = p.N >> 1;
#pragma unroll 1
          for (int c = half; c < 4; c += 2) {
            uint32_t rg[32], ru[32];
            const uint32_t ta = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                static_cast<uint32_t>(acc * Lay::kAccStride + c * 32);
            tmem_ld32(ta, rg);
            tmem_ld32(ta + 128, ru);
            const int col0 = nb * 128 + c * 32;
            float g[32], u[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              g[j] = __uint_as_float(rg[j]) * s;
              u[j] = __uint_as_float(ru[j]) * s;
            }
            if (p.bias) {
              add_bias32(g, p.bias + col0);
              add_bias32(u, p.bias + h + col0);
            }
            uint32_t w[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float lo = silu_bf16(bf16_round(g[2 * j])) * bf16_round(u[2 * j]);
              const float hi = silu_bf16(bf16_round(g[2 * j + 1])) * bf16_round(u[2 * j + 1]);
              w[j] = pack_bf16x2(lo, hi);
            }
            if (p.amax_out && row_ok) {
              uint32_t m2 = 0;
#pragma unroll
              for (int j = 0; j < 16; ++j) m2 = __vmaxu2(m2, w[j] & 0x7FFF7FFFu);
              amax_local = max(amax_local, max(m2 & 0xFFFFu, m2 >> 16));
            }
            store_bf16(w, col0);
          }
        }
      }
#pragma unroll 1
      for (int c = half; c < chunks; c += 2) {
        uint32_t r[32];
        tmem_ld32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                      static_cast<uint32_t>(acc * Lay::kAccStride + c * 32),
                  r);
        const int col0 = nb * BN + c * 32;
        if (col0 >= p.N) continue;                    // warp-uniform
        const int ncols = min(32, p.N - col0);        // 16 or 32 (N % 16 == 0)
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * s;
        if (p.bias) add_bias32(v, p.bias + col0, ncols);
        if (p.out_f32) {
          // two 16-column blocks of 64-byte rows, 64-byte swizzle
#pragma unroll
          for (int hb = 0; hb < 2; ++hb) {
            if (hb * 16 >= ncols) break;
            if (lane == 0) bulk_wait_read_1();
            __syncwarp();
            uint8_t* sb = stage_out + buf * Lay::kOutBufBytes;
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<float4*>(sb + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)) =
                  make_float4(v[hb * 16 + 4 * q], v[hb * 16 + 4 * q + 1], v[hb * 16 + 4 * q + 2],
                              v[hb * 16 + 4 * q + 3]);
            if (p.epilogue == QIK_EPI_SCATTER) {
              // 32 rows x 64 bytes: lane l stores 16-byte chunk (l & 3) of rows
              // (l >> 2) + 8 i, i.e. 8 contiguous 64-byte row pieces per store
              __syncwarp();
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int rr = (lane >> 2) + 8 * i, q = lane & 3;
                const int grow = row0 + rr;
                const float4 val =
                    *reinterpret_cast<const float4*>(sb + rr * 64 + ((q ^ ((rr >> 1) & 3)) << 4));
                if (grow < p.M) {
                  const int o = grow / p.scat_rows;
                  float* dst = p.scat_dst[o] + static_cast<int64_t>(grow - o * p.scat_rows) * p.N + col0 + hb * 16 + 4 * q;
                  *reinterpret_cast<float4*>(dst) = val;
                }
              }
              __syncwarp();
            } else {
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0 && row0 < p.M) {
                tma_store_2d(&tmC, col0 + hb * 16, row0, sb);
                bulk_commit_group();
              }
            }
            buf ^= 1;
          }
        } else {
          uint32_t w[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float lo = v[2 * j], hi = v[2 * j + 1];
            if (p.epilogue == QIK_EPI_GELU_TANH) {
              lo = gelu_tanh_f32(__bfloat162float(__float2bfloat16_rn(lo)));
              hi = gelu_tanh_f32(__bfloat162float(__float2bfloat16_rn(hi)));
            }
            w[j] = pack_bf16x2(lo, hi);
          }
          if (EK == kEkGate && row_ok) {
            // x + bf16(T * f) in bf16x2 arithmetic: the products and sums of bf16 values,
            // each rounded once, as the gated-residual kernel's fp32 arithmetic rounds them
            const int grow = row0 + lane, b = grow / p.gate_seq, sq = grow - b * p.gate_seq;
            const int t = b + ((p.gate_mask != nullptr && p.gate_mask[sq] == 0) ? p.gate_batch : 0);
            const uint4* xp = reinterpret_cast<const uint4*>(p.res_x + static_cast<int64_t>(grow) * p.res_ld + col0);
            const uint4* tp = reinterpret_cast<const uint4*>(p.gate_tab + static_cast<int64_t>(t) * p.gate_ld + col0);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              if (q * 8 < ncols) {
                const uint4 xv = __ldg(xp + q), tv = __ldg(tp + q);
                w[4 * q] = add_bf16x2(xv.x, mul_bf16x2(tv.x, w[4 * q]));
                w[4 * q + 1] = add_bf16x2(xv.y, mul_bf16x2(tv.y, w[4 * q + 1]));
                w[4 * q + 2] = add_bf16x2(xv.z, mul_bf16x2(tv.z, w[4 * q + 2]));
                w[4 * q + 3] = add_bf16x2(xv.w, mul_bf16x2(tv.w, w[4 * q + 3]));
              }
            }
          }
          if (p.amax_out && row_ok) {
            uint32_t m2 = 0;
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (2 * j < ncols) m2 = __vmaxu2(m2, w[j] & 0x7FFF7FFFu);
            amax_local = max(amax_local, max(m2 & 0xFFFFu, m2 >> 16));
          }
          store_bf16(w, col0);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (TWO_SM)
          mbar_arrive_remote(mapa_shared(&tempty[acc], 0));  // the leader's accumulator barrier
        else
          mbar_arrive(&tempty[acc]);
      }
      if (p.epilogue == QIK_EPI_SCATTER) {
        // the tile's rows of this CTA are stored by all epilogue warps; then one thread
        // releases them at system scope (cumulative over the barrier) and counts the
        // tile at the owner of the tile's rows (tiles never straddle owners)
        named_bar_sync(1, 32 * kGemmEpiWarps);
        if (warp == 2 && lane == 0) {
          __threadfence_system();
          atomicAdd_system(p.scat_cnt[(mb * kTileM) / p.scat_rows], 1u);
        }
      }
    }
    if (lane == 0) bulk_wait_all();
    if (p.amax_out) {
      amax_local = __reduce_max_sync(0xffffffffu, amax_local);
      if (lane == 0 && amax_local != 0u) atomicMax(p.amax_out, amax_local << 16);
    }
  }

  tc_fence_before();
  __syncthreads();
  // the leader's MMAs read the peer's shared memory and write its tensor memory: neither
  // CTA frees either before both are done
  if constexpr (TWO_SM) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (TWO_SM)
      tmem_dealloc_cg2(tmem_base, Lay::kTmemCols);
    else
      tmem_dealloc(tmem_base, Lay::kTmemCols);
  }
}

// Tile configurations (QIK_GEMM_TILE_* in qik.h): CTA pairs computing 256 x 256 tiles,
// or single CTAs with 128 x BN tiles (BN = 256, 128 or 64).
//
// Shape -> tile configuration, from the configs[4] sweep with every configuration
// forced: CTA pairs from M = 257 up (but 128 x 256 single-CTA tiles for 257-1024 rows
// of an output at most 3072 wide), and at M = 129-256 once N >= 12288; at M = 129-256
// with a narrower N, 128 x 128 single-CTA tiles (more CTAs on the same work) win; at
// most 128 rows, a single 128-row tile spans M and the N tiles spread the weight
// stream over the SMs.  Narrower CTA-pair tiles (256 x 240, 256 x 192), chosen to fill
// the last wave that 256-wide tiles leave partly empty, were built and measured slower
// at every configs[4] shape and at the FFN's (4352 x 12288: 120.7 and 139.3 us against
// 116.4): a 240-wide tile took about as long as a 256-wide one, and 192-wide tiles read
// ~17% more operand bytes per FLOP.
// At most 16 rows (the DiT's timestep-modulation linear: M = 2), the operands swap
// (QIK_GEMM_TILE_SWAP_16): 128 weight rows per tile against the 16-row activation tile,
// 18 KB per pipeline stage instead of 32 KB, so 11 stages of the weight stream are in
// flight per SM instead of 6; the scatter (tensor-parallel) epilogue keeps the
// untransposed tiles.
static int gemm_pick_cfg(int64_t M, int64_t N, bool scatter = false) {
  // up to 1024 rows of a narrow output (N <= 3072), 128 x 256 single-CTA tiles: the same
  // CTA count as pairs at M = 1024 and measured faster there (18.5 vs 20.5 us)
  if (M > 2 * kGemmBM && M <= 8 * kGemmBM && N <= 3072 && !scatter) return QIK_GEMM_TILE_SINGLE_256;
  if (M > 2 * kGemmBM) return QIK_GEMM_TILE_PAIR_256;
  if (M > kGemmBM) return N >= 12288 ? QIK_GEMM_TILE_PAIR_256 : QIK_GEMM_TILE_SINGLE_128;
  if (M <= 16 && !scatter) return QIK_GEMM_TILE_SWAP_16;
  return (N + 127) / 128 >= sm_count() / 2 ? QIK_GEMM_TILE_SINGLE_128 : QIK_GEMM_TILE_SINGLE_64;
}

// Raster group (row tiles per group, tile_coords).  Measured on the configs[4] shapes
// and the DiT block's (1 x B200, groups of 1, 2, 4, 8 and 16 row tiles forced): for a B
// of 18432 x 3072 (56.6 MB, more than L2 keeps from one wave to the next in row-major
// order) groups of 16 gain 2-5% (16384 x 18432 677.5 -> 644.9 us, 9472 x 18432 374.2
// -> 359.9, 4352 x 18432 171.3 -> 167.1); where B is smaller they are within 1% either
// way but read more: the FFN's down projection (4352 x 3072 x 12288) ran faster alone
// with groups of 16 (113.2 against 124.5 us, L2 flushed) yet read 200 MB of DRAM instead
// of 118 MB, and inside the FFN chain, whose pack leaves A in L2, it was no faster.
static int gemm_pick_raster(int64_t N, int64_t K) { return N * K > (int64_t{48} << 20) ? 16 : 1; }

template <int BN, int STAGES, bool TWO_SM, int EK = kEkPlain>
static int launch_gemm(const uint8_t* A, const uint8_t* B, const GemmParams& p, int64_t lda, int64_t ldb,
                       cudaStream_t st, bool pdl) {
  using Lay = GemmLayout<BN, STAGES, TWO_SM>;
  constexpr int kBRows = TWO_SM ? BN / 2 : BN;  // rows of B each CTA loads per stage
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, static_cast<uint64_t>(p.K),
                        static_cast<uint64_t>(p.M), static_cast<uint64_t>(lda), kGemmBK, kGemmBM,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, static_cast<uint64_t>(p.K), static_cast<uint64_t>(p.N),
                    static_cast<uint64_t>(ldb), kGemmBK, kBRows, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  CUtensorMap tc;
  // the output [rows, cols]: the kernel's [M, N], or [N, M] in the transposed tiny-M
  // form (whose epilogue stores without the map)
  const uint64_t c_cols = static_cast<uint64_t>(BN == 16 ? p.M : (p.epilogue == QIK_EPI_SWIGLU ? p.N / 2 : p.N));
  const uint64_t c_rows = static_cast<uint64_t>(BN == 16 ? p.N : p.M);
  if (p.out_f32)
    rc = make_tmap_2d(&tc, p.C, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, c_cols, c_rows, static_cast<uint64_t>(p.ldc) * 4, 16,
                      32, CU_TENSOR_MAP_SWIZZLE_64B);
  else
    rc = make_tmap_2d(&tc, p.C, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, c_cols, c_rows, static_cast<uint64_t>(p.ldc) * 2, 32,
                      32, CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  static std::once_flag attr_once[64];
  int dev = 0;
  QIK_TRY_CUDA(cudaGetDevice(&dev));
  QIK_REQUIRE(dev >= 0 && dev < 64, "qik_fp8_gemm: device ordinal %d out of range", dev);
  cudaError_t attr_rc = cudaSuccess;
  std::call_once(attr_once[dev], [&] {
    attr_rc = cudaFuncSetAttribute(fp8_gemm_kernel<BN, STAGES, TWO_SM, EK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   Lay::kSmemBytes);
  });
  QIK_TRY_CUDA(attr_rc);
  constexpr int kTileM = TWO_SM ? 2 * kGemmBM : kGemmBM;
  const int tiles = ((p.M + kTileM - 1) / kTileM) * ((p.N + BN - 1) / BN);
  if constexpr (TWO_SM) {
    // persistent CTA pairs (clusters of 2), at most one CTA per SM
    const int pairs = min(tiles, sm_count() / 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = Lay::kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    QIK_TRY_CUDA(cudaLaunchKernelEx(&cfg, fp8_gemm_kernel<BN, STAGES, TWO_SM, EK>, ta, tb, tc, p));
  } else {
    const int grid = min(tiles, sm_count());
    QIK_TRY_CUDA(launch_kernel(fp8_gemm_kernel<BN, STAGES, TWO_SM, EK>, dim3(grid), dim3(kGemmThreads), Lay::kSmemBytes,
                               st, pdl, ta, tb, tc, p));
  }
  return check_launch("fp8_gemm_kernel");
}

int launch_fp8_gemm_ex(const uint8_t* A, const uint8_t* B, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                       const float* scale_a, const float* scale_b, const void* bias, void* C, int64_t ldc,
                       int out_dtype, int epilogue, uint32_t* amax_out, int* status, cudaStream_t stream, bool pdl,
                       const GemmParams* scatter, int tile_cfg = QIK_GEMM_TILE_AUTO) {
  QIK_REQUIRE(M >= 0 && N >= 0 && K >= 0, "qik_fp8_gemm: negative size");
  if (M == 0 || N == 0) return QIK_OK;
  QIK_REQUIRE(K > 0, "qik_fp8_gemm: K must be positive");
  QIK_REQUIRE(M <= (1ll << 31) - 1 && N <= (1ll << 31) - 1 && K <= (1ll << 31) - 1, "qik_fp8_gemm: size above 2^31");
  QIK_REQUIRE(A && B && C && scale_a && scale_b, "qik_fp8_gemm: NULL operand");
  QIK_REQUIRE(K % 16 == 0, "qik_fp8_gemm: K=%lld must be a multiple of 16", (long long)K);
  QIK_REQUIRE(lda >= K && lda % 16 == 0 && ldb >= K && ldb % 16 == 0,
              "qik_fp8_gemm: lda/ldb must be >= K and multiples of 16 bytes");
  QIK_REQUIRE(aligned16(A) && aligned16(B) && aligned16(C), "qik_fp8_gemm: A, B, C must be 16-byte aligned");
  QIK_REQUIRE(N % 16 == 0, "qik_fp8_gemm: N=%lld must be a multiple of 16", (long long)N);
  const bool swiglu = epilogue == QIK_EPI_SWIGLU;
  const int64_t c_cols = swiglu ? N / 2 : N;
  QIK_REQUIRE(ldc >= c_cols && ldc % 8 == 0, "qik_fp8_gemm: ldc must be >= the output width and a multiple of 8");
  QIK_REQUIRE(out_dtype == QIK_DTYPE_BF16 || out_dtype == QIK_DTYPE_F32, "qik_fp8_gemm: out_dtype must be BF16/F32");
  const bool rms = epilogue == QIK_EPI_RMS_ROPE;
  const bool gate = epilogue == QIK_EPI_GATE_RES;
  QIK_REQUIRE(epilogue == QIK_EPI_SCALE || epilogue == QIK_EPI_GELU_TANH ||
                  (epilogue == QIK_EPI_SCATTER && scatter && out_dtype == QIK_DTYPE_F32 && !bias) ||
                  (swiglu && !scatter) ||
                  (rms && scatter && scatter->rms_cols > 0 && out_dtype == QIK_DTYPE_BF16 && !amax_out) ||
                  (gate && scatter && scatter->res_x && out_dtype == QIK_DTYPE_BF16),
              "qik_fp8_gemm: unknown epilogue (QIK_EPI_RMS_ROPE and QIK_EPI_GATE_RES only through their entry "
              "points)");
  QIK_REQUIRE(!swiglu || (N % 256 == 0 && out_dtype == QIK_DTYPE_BF16),
              "qik_fp8_gemm: the SwiGLU epilogue needs N %% 256 == 0 (N=%lld) and BF16 output", (long long)N);
  QIK_REQUIRE(!(out_dtype == QIK_DTYPE_F32 && ((epilogue != QIK_EPI_SCALE && epilogue != QIK_EPI_SCATTER) || amax_out)),
              "qik_fp8_gemm: GELU and amax need BF16 output");
  QIK_REQUIRE(!bias || aligned16(bias), "qik_fp8_gemm: bias must be 16-byte aligned");
  GemmParams p;
  if (scatter)
    p = *scatter;
  else
    memset(&p, 0, sizeof(p));
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.scale_a = scale_a;
  p.scale_b = scale_b;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.C = C;
  p.ldc = ldc;
  p.out_f32 = out_dtype == QIK_DTYPE_F32;
  p.epilogue = epilogue;
  p.amax_out = amax_out;
  p.status = status;
  const int sel = tile_cfg & 0xFF;
  // SwiGLU: a CTA-pair tile holds the gate and the up columns of the same 128 outputs
  const int cfg = (swiglu || rms) ? QIK_GEMM_TILE_PAIR_256
                                  : (sel == QIK_GEMM_TILE_AUTO ? gemm_pick_cfg(M, N, scatter != nullptr) : sel);
  QIK_REQUIRE(!swiglu || sel == QIK_GEMM_TILE_AUTO || sel == QIK_GEMM_TILE_PAIR_256,
              "qik_fp8_gemm: the SwiGLU epilogue runs on CTA-pair tiles only (tile configuration %d)", sel);
  const int raster = (tile_cfg >> 8) & 0xFF;
  p.group_m = raster != 0 ? raster : gemm_pick_raster(N, K);
  const int ek = swiglu ? kEkSwiglu : rms ? kEkRms : gate ? kEkGate : kEkPlain;
  switch (cfg) {
    case QIK_GEMM_TILE_PAIR_256:
      switch (ek) {
        case kEkSwiglu:
          return launch_gemm<256, 6, true, kEkSwiglu>(A, B, p, lda, ldb, stream, pdl);
        case kEkRms:
          return launch_gemm<256, 6, true, kEkRms>(A, B, p, lda, ldb, stream, pdl);
        case kEkGate:
          return launch_gemm<256, 6, true, kEkGate>(A, B, p, lda, ldb, stream, pdl);
        default:
          return launch_gemm<256, 6, true>(A, B, p, lda, ldb, stream, pdl);
      }
    case QIK_GEMM_TILE_SINGLE_128:
      return ek == kEkGate ? launch_gemm<128, 6, false, kEkGate>(A, B, p, lda, ldb, stream, pdl)
                           : launch_gemm<128, 6, false>(A, B, p, lda, ldb, stream, pdl);
    case QIK_GEMM_TILE_SINGLE_64:
      return ek == kEkGate ? launch_gemm<64, 8, false, kEkGate>(A, B, p, lda, ldb, stream, pdl)
                           : launch_gemm<64, 8, false>(A, B, p, lda, ldb, stream, pdl);
    case QIK_GEMM_TILE_SINGLE_256:
      return ek == kEkGate ? launch_gemm<256, 4, false, kEkGate>(A, B, p, lda, ldb, stream, pdl)
                           : launch_gemm<256, 4, false>(A, B, p, lda, ldb, stream, pdl);
    case QIK_GEMM_TILE_SWAP_16: {
      // C^T = B . A^T: the weights are the tile rows, the (at most 16) activation rows
      // the tile columns; the epilogue stores C untransposed
      QIK_REQUIRE(M <= 16 && !scatter, "qik_fp8_gemm: the swapped tiny-M configuration needs M <= 16, got %lld",
                  static_cast<long long>(M));
      GemmParams q = p;
      q.M = p.N;
      q.N = p.M;
      q.group_m = 1;
      return launch_gemm<16, 11, false>(B, A, q, ldb, lda, stream, pdl);
    }
    default:
      return set_error(QIK_ERR_INVALID, "qik_fp8_gemm: unknown tile configuration %d", cfg);
  }
}

int launch_fp8_gemm(const uint8_t* A, const uint8_t* B, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                    const float* scale_a, const float* scale_b, const void* bias, void* C, int64_t ldc, int out_dtype,
                    int epilogue, uint32_t* amax_out, int* status, cudaStream_t stream, bool pdl, bool keep_out_l2) {
  if (!keep_out_l2)
    return launch_fp8_gemm_ex(A, B, M, N, K, lda, ldb, scale_a, scale_b, bias, C, ldc, out_dtype, epilogue, amax_out,
                              status, stream, pdl, nullptr, QIK_GEMM_TILE_AUTO);
  GemmParams extra;
  memset(&extra, 0, sizeof(extra));
  extra.keep_out_l2 = 1;
  // (an extras block keeps the scatter-safe tile choice: no operand-swapped tiny-M tiles)
  return launch_fp8_gemm_ex(A, B, M, N, K, lda, ldb, scale_a, scale_b, bias, C, ldc, out_dtype, epilogue, amax_out,
                            status, stream, pdl, &extra, QIK_GEMM_TILE_AUTO);
}

}  // namespace qik

namespace qik {
// Tile height and width of the configuration launch_fp8_gemm picks for (M, N).
static void gemm_tile_shape(int64_t M, int64_t N, int* tile_m, int* tile_n, int* ctas_per_tile) {
  const int cfg = gemm_pick_cfg(M, N, true);  // the scatter epilogue's tiles
  const bool pair = cfg == QIK_GEMM_TILE_PAIR_256;
  *tile_m = pair ? 2 * kGemmBM : kGemmBM;
  *tile_n = (pair || cfg == QIK_GEMM_TILE_SINGLE_256) ? 256 : (cfg == QIK_GEMM_TILE_SINGLE_128 ? 128 : 64);
  *ctas_per_tile = pair ? 2 : 1;
}
}  // namespace qik

extern "C" int64_t qik_fp8_gemm_scatter_signals(int64_t M, int64_t N, int64_t rows_per_owner, int owner) {
  if (M <= 0 || N <= 0 || rows_per_owner <= 0 || owner < 0) return 0;
  int tm, tn, cpt;
  qik::gemm_tile_shape(M, N, &tm, &tn, &cpt);
  const int64_t lo = static_cast<int64_t>(owner) * rows_per_owner;
  const int64_t hi = lo + rows_per_owner < M ? lo + rows_per_owner : M;
  if (hi <= lo) return 0;
  // tiles whose first row lies in [lo, hi): rows_per_owner is a multiple of the tile height
  const int64_t tiles_m = (hi - lo + tm - 1) / tm;
  return tiles_m * ((N + tn - 1) / tn) * cpt;
}

extern "C" int qik_fp8_gemm_scatter(const uint8_t* A, const uint8_t* B, int64_t M, int64_t N, int64_t K, int64_t lda,
                                    int64_t ldb, const float* scale_a, const float* scale_b, int world,
                                    int64_t rows_per_owner, float* const* dst, uint32_t* const* cnt, int* status,
                                    void* stream) {
  using namespace qik;
  QIK_REQUIRE(world >= 1 && world <= QIK_TP_MAX_WORLD, "qik_fp8_gemm_scatter: world %d outside 1..%d", world,
              QIK_TP_MAX_WORLD);
  QIK_REQUIRE(dst && cnt, "qik_fp8_gemm_scatter: NULL dst / cnt array");
  QIK_REQUIRE(rows_per_owner > 0 && rows_per_owner % (2 * kGemmBM) == 0 && rows_per_owner * world >= M,
              "qik_fp8_gemm_scatter: rows per owner must be a positive multiple of %d covering M", 2 * kGemmBM);
  QIK_REQUIRE(M <= (1ll << 31) - 1 && N <= (1ll << 31) - 1, "qik_fp8_gemm_scatter: size above 2^31");
  for (int o = 0; o < world; ++o)
    QIK_REQUIRE(dst[o] && cnt[o] && aligned16(dst[o]), "qik_fp8_gemm_scatter: dst[%d] / cnt[%d] NULL or unaligned",
                o, o);
  // the rest of the checks and the launch are qik_fp8_gemm's, with fp32 output
  GemmParams extra;
  memset(&extra, 0, sizeof(extra));
  for (int o = 0; o < world; ++o) {
    extra.scat_dst[o] = dst[o];
    extra.scat_cnt[o] = cnt[o];
  }
  extra.scat_rows = static_cast<int>(rows_per_owner);
  return launch_fp8_gemm_ex(A, B, M, N, K, lda, ldb, scale_a, scale_b, nullptr, dst[0], N, QIK_DTYPE_F32,
                            QIK_EPI_SCATTER, nullptr, status, static_cast<cudaStream_t>(stream), false, &extra);
}

extern "C" int qik_fp8_gemm_qkv_rms_rope(const uint8_t* A, const uint8_t* B, int64_t M, int64_t K, int64_t lda,
                                         int64_t ldb, const float* scale_a, const float* scale_b, const void* bias,
                                         void* C, int64_t ldc, int heads, int head_dim, const float* w_q,
                                         const float* w_k, const float* rope_cos, const float* rope_sin, int64_t seq,
                                         float eps, int* status, void* stream) {
  using namespace qik;
  QIK_REQUIRE(head_dim == 128, "qik_fp8_gemm_qkv_rms_rope: head_dim must be 128, got %d", head_dim);
  QIK_REQUIRE(heads >= 1 && heads <= 4096, "qik_fp8_gemm_qkv_rms_rope: heads %d out of range", heads);
  QIK_REQUIRE(w_q && w_k && rope_cos && rope_sin, "qik_fp8_gemm_qkv_rms_rope: NULL norm weight / rotary table");
  QIK_REQUIRE(aligned16(w_q) && aligned16(w_k) && aligned16(rope_cos) && aligned16(rope_sin),
              "qik_fp8_gemm_qkv_rms_rope: norm weights and rotary tables must be 16-byte aligned");
  QIK_REQUIRE(seq >= 1 && seq <= (1ll << 31) - 1 && M % seq == 0,
              "qik_fp8_gemm_qkv_rms_rope: M=%lld must be a multiple of seq=%lld", (long long)M, (long long)seq);
  GemmParams extra;
  memset(&extra, 0, sizeof(extra));
  extra.rms_w[0] = w_q;
  extra.rms_w[1] = w_k;
  extra.rope_cos = rope_cos;
  extra.rope_sin = rope_sin;
  extra.rope_seq = static_cast<int>(seq);
  extra.rms_cols = 2 * heads * head_dim;
  extra.rms_eps = eps;
  const int64_t N = 3ll * heads * head_dim;
  return launch_fp8_gemm_ex(A, B, M, N, K, lda, ldb, scale_a, scale_b, bias, C, ldc, QIK_DTYPE_BF16, QIK_EPI_RMS_ROPE,
                            nullptr, status, static_cast<cudaStream_t>(stream), true, &extra, QIK_GEMM_TILE_PAIR_256);
}

extern "C" int qik_fp8_gemm_gate_residual(const uint8_t* A, const uint8_t* B, int64_t M, int64_t N, int64_t K,
                                          int64_t lda, int64_t ldb, const float* scale_a, const float* scale_b,
                                          const void* bias, const void* x, int64_t ldx, const void* gate_table,
                                          int64_t ldt, const uint8_t* target_mask, int64_t batch, int64_t seq,
                                          void* C, int64_t ldc, int* status, void* stream) {
  using namespace qik;
  QIK_REQUIRE(x && gate_table, "qik_fp8_gemm_gate_residual: NULL residual / gate table");
  QIK_REQUIRE(aligned16(x) && aligned16(gate_table) && ldx % 8 == 0 && ldt % 8 == 0 && ldx >= N && ldt >= N,
              "qik_fp8_gemm_gate_residual: residual and gate table must be 16-byte aligned with row pitches >= N "
              "and multiples of 8");
  QIK_REQUIRE(batch >= 1 && seq >= 1 && batch * seq == M && M <= (1ll << 31) - 1,
              "qik_fp8_gemm_gate_residual: M=%lld is not batch=%lld x seq=%lld", (long long)M, (long long)batch,
              (long long)seq);
  GemmParams extra;
  memset(&extra, 0, sizeof(extra));
  extra.res_x = static_cast<const uint16_t*>(x);
  extra.res_ld = ldx;
  extra.gate_tab = static_cast<const uint16_t*>(gate_table);
  extra.gate_ld = ldt;
  extra.gate_mask = target_mask;
  extra.gate_seq = static_cast<int>(seq);
  extra.gate_batch = static_cast<int>(batch);
  return launch_fp8_gemm_ex(A, B, M, N, K, lda, ldb, scale_a, scale_b, bias, C, ldc, QIK_DTYPE_BF16, QIK_EPI_GATE_RES,
                            nullptr, status, static_cast<cudaStream_t>(stream), true, &extra, QIK_GEMM_TILE_AUTO);
}

extern "C" int qik_fp8_gemm(const uint8_t* A, const uint8_t* B, int64_t M, int64_t N, int64_t K, int64_t lda,
                            int64_t ldb, const float* scale_a, const float* scale_b, const void* bias, void* C,
                            int64_t ldc, int out_dtype, int epilogue, uint32_t* amax_out, int* status,
                            void* stream) {
  return qik::launch_fp8_gemm(A, B, M, N, K, lda, ldb, scale_a, scale_b, bias, C, ldc, out_dtype, epilogue, amax_out,
                              status, static_cast<cudaStream_t>(stream), true);
}

extern "C" int qik_fp8_gemm_tiled(const uint8_t* A, const uint8_t* B, int64_t M, int64_t N, int64_t K, int64_t lda,
                                  int64_t ldb, const float* scale_a, const float* scale_b, const void* bias, void* C,
                                  int64_t ldc, int out_dtype, int epilogue, uint32_t* amax_out, int tile_cfg,
                                  int* status, void* stream) {
  const int sel = tile_cfg & 0xFF;
  QIK_REQUIRE((tile_cfg & ~0xFFFF) == 0 &&
                  (sel == QIK_GEMM_TILE_AUTO || sel == QIK_GEMM_TILE_PAIR_256 || sel == QIK_GEMM_TILE_SINGLE_256 ||
                   sel == QIK_GEMM_TILE_SINGLE_128 || sel == QIK_GEMM_TILE_SINGLE_64 || sel == QIK_GEMM_TILE_SWAP_16),
              "qik_fp8_gemm_tiled: unknown tile configuration %d", tile_cfg);
  return qik::launch_fp8_gemm_ex(A, B, M, N, K, lda, ldb, scale_a, scale_b, bias, C, ldc, out_dtype, epilogue,
                                 amax_out, status, static_cast<cudaStream_t>(stream), true, nullptr, tile_cfg);
}
