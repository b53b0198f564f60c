// qik_attn.cu -- block-causal flash attention over [prefix slab ; fresh K/V] on the
// sm_100a tensor core.
//
// Semantics of block_causal_flash_attention / _qwen21_attn_fwd
// (qwen_image_kernel/triton_attention.py:35-260): query row r of (b, h) attends to
// the keys kv of the virtual concatenation [cache (P keys) ; fresh (SN keys)] with
// kv <= L[r] (all keys when UNIFORM) and key_valid[b, kv] != 0 (when given);
// softmax in base 2 with the scores scaled by sm_scale * log2(e); P is rounded to
// the tensors' type (bf16, or fp16 under QIK_ATTN_F16) before P.V; fp32
// accumulation; rows with no allowed key are 0.
// e4m3 slab V (triton_attention.py:154-159, which rounds fl32(v8) * scale[b, h] to
// bf16 per element): here the slab tiles multiply e4m3-exact f16 V by f16 P (a
// finer rounding of P than bf16) and the per-(b, h) scale multiplies the fp32
// accumulator once at the slab -> fresh boundary, i.e. the exact fp32 dequant
// product fl32(v8) * scale; the difference to the reference kernel's bf16 rounding
// of each dequantized V element is below half a bf16 ulp of V.
//
// One CTA per (256-query block, b, h): two 128-row query tiles, A and B, share every
// K/V tile, and each has its own 8 softmax warps, so the tensor core computes one
// tile's S and P.V while the other tile's softmax runs.
//   warp 0      TMA producer: Q_A and Q_B once (64-column halves, 128-byte swizzle),
//               K tiles into a 2-stage ring (freed once S_A and S_B are computed), V
//               tiles (bf16, or e4m3 raw for the fp8 slab) into a 2-stage ring (freed
//               after P_B.V), V lagging K by one tile;
//   warp 1      MMA issuer (one thread), per key tile t:
//                 O_A += P_A(t) V_t ; S_A(t+1) = Q_A K_{t+1}^T ;
//                 O_B += P_B(t) V_t ; S_B(t+1) = Q_B K_{t+1}^T
//               tcgen05.mma runs in issue order and tcgen05.commit tracks every
//               earlier MMA of the thread, so when S_g(t+1) is complete, P_g(t).V has
//               been consumed: P_g(t+1) can overwrite S_g's columns and O_g can be
//               rescaled without another barrier;
//   warps 2-3   e4m3 -> f16 V converters for slab tiles when V is fp8 (exact);
//   warps 4-11  softmax of tile A, warps 12-19 softmax of tile B: two threads per
//               query row (16x32bx2 TMEM accesses), each with 64 of its 128 scores,
//               so a tile's softmax takes half the time of one thread per row and
//               fits inside the other tile's MMAs; each thread reads its half of
//               S_g(t) from TMEM, masks, takes the row max with one shuffle, keeps an
//               online half-row sum (O_g is rescaled in TMEM only when the running
//               max grows by more than 2^8, which leaves the final O/l unchanged),
//               writes its half of P_g(t) as bf16 over the first 32 of its own S
//               columns; finally O_g / l -> bf16 -> global, each thread 64 columns.
// TMEM columns: S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512); P_g(keys 0-63)
// over S_g columns 0-31, P_g(keys 64-127) over S_g columns 64-95.
// CTAs are numbered heaviest-first (the last query blocks, which see the most keys
// under a block-causal mask, start first) so the short blocks fill the tail.
#include <mutex>

#include "qik_device.cuh"
#include "qik_host.h"

namespace qik {

constexpr int kAttnBM = 128;                        // query rows per tile (one TMEM lane each)
constexpr int kAttnTiles = 2;                       // query tiles per CTA
constexpr int kAttnRows = kAttnBM * kAttnTiles;     // query rows per CTA
constexpr int kAttnBN = 128;
constexpr int kAttnD = 128;
constexpr int kAttnHalf = kAttnBN / 2;              // scores per softmax thread: half a row
constexpr int kAttnSoftmaxWarps = 8;                // per query tile: two threads per row
constexpr int kAttnThreads = 128 + 32 * kAttnSoftmaxWarps * kAttnTiles;  // producer, MMA, 2 converters, softmax
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O when the max grows by > 2^8
// Softmax exponentials: pairs j >= kPolyFromPair of a half row (on tiles where every
// key is allowed) use the FMA-pipe 2^x, the others MUFU ex2 (9 of the 32 pairs, the
// share measured best for the two pipes).
constexpr int kPolyFromPair = 23;

struct AttnSmem {
  static constexpr int kQ = 0;                          // per tile 32 KB: two 16 KB halves (d 0-63, 64-127)
  static constexpr int kKStages = 2;
  static constexpr int kVStages = 2;
  static constexpr int kK0 = kAttnTiles * 32768;        // K ring: 2 x 32 KB
  static constexpr int kV0 = kK0 + kKStages * 32768;    // V ring: 2 x 32 KB (bf16)
  static constexpr int kV80 = kV0 + kVStages * 32768;   // raw e4m3 V: 2 x 16 KB
  static constexpr int kBar = kV80 + kVStages * 16384;
  static constexpr int kBytes = kBar + 256 + 1024;      // barriers + alignment slack
};
static_assert(AttnSmem::kBytes <= 232448, "attention shared memory above the 227 KB per-CTA limit");

struct AttnDev {
  const int32_t* L;
  const uint8_t* key_valid;
  const float* v_scale;
  uint16_t* out;  // bf16 or fp16 bits
  int64_t o_sb, o_ss, o_sh, kv_sb;
  int SQ, SN, P, H;
  float qk_scale_log2;
  int flags;
  int* status;
  uint32_t* amax_out;
};

// Two boxes of 64 d-columns x 128 keys (rows) of one (b, h).
__device__ __forceinline__ void load_bf16_tile(const CUtensorMap* tm, void* dst, int key0, int h, int b,
                                               uint64_t* bar) {
  tma_load_4d(dst, tm, 0, key0, h, b, bar);
  tma_load_4d(static_cast<uint8_t*>(dst) + 16384, tm, 64, key0, h, b, bar);
}

// P half row of one 128-key tile: the thread's 64 scores (columns 64 hc .. 64 hc + 63
// of its row), p = 2^(s * scale - m) computed in pairs (f32x2), packed (f16 for
// fp8-slab tiles, else bf16) and written to TMEM at tP with the 16x32bx2 shape: the
// hc = 0 thread's 32 packed words at columns 0-31 of S_g, the hc = 1 thread's at 64-95,
// each over scores that thread has already read.  Returns the half row's fp32 sum.
// kPoly (tiles where every key of the row is allowed): pairs j >= kPolyFromPair take
// 2^x on the FMA pipe (exp2_poly2), the rest MUFU ex2, so the two pipes share the
// exponentials.
template <bool kPoly, bool kF16>
__device__ __forceinline__ float softmax_half_row(const float (&sv)[kAttnHalf], float scale, float neg_m,
                                                  uint32_t tP) {
  const uint64_t sc2 = f2_pack(scale, scale), nm2 = f2_pack(neg_m, neg_m);
  uint64_t acc[2] = {0ull, 0ull};  // (0.f, 0.f) pairs
  uint32_t pk[kAttnHalf / 2];
#pragma unroll
  for (int j = 0; j < kAttnHalf / 2; ++j) {
    const uint64_t x2 = ffma2(f2_pack(sv[2 * j], sv[2 * j + 1]), sc2, nm2);
    uint64_t p2;
    if (kPoly && j >= kPolyFromPair) {
      p2 = exp2_poly2(x2);
    } else {
      float x0, x1;
      f2_unpack(x2, x0, x1);
      p2 = f2_pack(ex2(x0), ex2(x1));
    }
    acc[j & 1] = fadd2(acc[j & 1], p2);
    float p0, p1;
    f2_unpack(p2, p0, p1);
    pk[j] = kF16 ? pack_f16x2(p0, p1) : pack_bf16x2(p0, p1);
  }
  __syncwarp();
  tmem_st_2x32(tP, pk);
  float a0, a1, b0, b1;
  f2_unpack(acc[0], a0, a1);
  f2_unpack(acc[1], b0, b1);
  return (a0 + a1) + (b0 + b1);
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_ck,
                    const __grid_constant__ CUtensorMap tm_cv, const AttnDev a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + AttnSmem::kBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* k_empty = bars + 3;   // [2] K stage free (after S_A and S_B)
  uint64_t* v_full = bars + 5;    // [2] V bf16 ready (TMA or converters)
  uint64_t* v8_full = bars + 7;   // [2] raw e4m3 V landed
  uint64_t* v_empty = bars + 9;   // [2] V stage free (after P_B.V)
  uint64_t* s_full = bars + 11;   // [tile] S_g(t) computed (and everything before it)
  uint64_t* p_full = bars + 13;   // [tile] P_g(t) written (its 8 softmax warps)
  uint64_t* o_full = bars + 15;   // [tile] last P_g.V done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* lmax_slot = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = (gridDim.y - 1 - blockIdx.y) * kAttnRows;  // heaviest-first
  const int bh = blockIdx.x;
  const int b = bh / a.H, h = bh % a.H;
  const bool has_cache = (a.flags & QIK_ATTN_HAS_CACHE) && a.P > 0;
  const bool uniform = (a.flags & QIK_ATTN_UNIFORM) != 0;
  const bool v_fp8 = has_cache && (a.flags & QIK_ATTN_V_FP8);
  const bool has_kv = (a.flags & QIK_ATTN_HAS_KEY_VALID) != 0;
  const bool f16 = (a.flags & QIK_ATTN_F16) != 0;  // fp16 tensors: f16 MMAs, P and output
  const int P = has_cache ? a.P : 0;
  const int kv_total = P + a.SN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v8_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], kAttnSoftmaxWarps);
      mbar_init(&o_full[s], 1);
    }
    *abort_flag = 0;
    *lmax_slot = -1;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // launched as a programmatic dependent: everything above touches no global memory;
  // the predecessor's results are read from here on
  pdl_wait();
  // per-row limits; the largest L of the block decides how many key tiles exist
  int my_L = -1;
  if (warp >= 4) {
    const int sw = warp - 4;  // softmax warp: tile sw / 8, rows 32 (sw % 4) + 16 ((sw / 4) % 2) + lane % 16
    const int r = m0 + (sw >> 3) * kAttnBM + (sw & 3) * 32 + ((sw >> 2) & 1) * 16 + (lane & 15);
    if (r < a.SQ) my_L = uniform ? kv_total - 1 : min(__ldg(a.L + r), kv_total - 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp >= 4) {
    const int wmax = __reduce_max_sync(0xffffffffu, my_L);
    if (lane == 0) atomicMax(lmax_slot, wmax);
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int lmax = *lmax_slot;
  const int tiles_slab_all = (P + kAttnBN - 1) / kAttnBN;
  const int n_slab = lmax < 0 ? 0 : min(tiles_slab_all, lmax / kAttnBN + 1);
  const int n_fresh = lmax < P ? 0 : min((a.SN + kAttnBN - 1) / kAttnBN, (lmax - P) / kAttnBN + 1);
  const int n_tiles = n_slab + n_fresh;

  uint8_t* sQ = smem + AttnSmem::kQ;
  auto k_ptr = [&](int s) { return smem + AttnSmem::kK0 + s * 32768; };
  auto v_ptr = [&](int s) { return smem + AttnSmem::kV0 + s * 32768; };
  auto v8_ptr = [&](int s) { return smem + AttnSmem::kV80 + s * 16384; };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n_tiles > 0) {
      tma_prefetch_desc(&tm_q);
      mbar_arrive_expect_tx(q_full, 32768 * kAttnTiles);
      for (int g = 0; g < kAttnTiles; ++g) load_bf16_tile(&tm_q, sQ + g * 32768, m0 + g * kAttnBM, h, b, q_full);
      // step u: K of tile u, then V of tile u - 1
      for (int u = 0; u <= n_tiles; ++u) {
        if (u < n_tiles) {
          const int ks = u & 1;
          const uint32_t kph = (u >> 1) & 1;
          if (!mbar_wait(&k_empty[ks], kph ^ 1u, abort_flag, a.status)) break;
          const bool slab = u < n_slab;
          const int key0 = slab ? u * kAttnBN : (u - n_slab) * kAttnBN;
          mbar_arrive_expect_tx(&k_full[ks], 32768);
          load_bf16_tile(slab ? &tm_ck : &tm_k, k_ptr(ks), key0, h, b, &k_full[ks]);
        }
        const int t = u - 1;
        if (t >= 0) {
          const int vs = t & 1;
          const uint32_t vph = (t >> 1) & 1;
          if (!mbar_wait(&v_empty[vs], vph ^ 1u, abort_flag, a.status)) break;
          const bool slab = t < n_slab;
          const int key0 = slab ? t * kAttnBN : (t - n_slab) * kAttnBN;
          if (slab && v_fp8) {
            mbar_arrive_expect_tx(&v8_full[vs], 16384);
            tma_load_4d(v8_ptr(vs), &tm_cv, 0, key0, h, b, &v8_full[vs]);
          } else {
            mbar_arrive_expect_tx(&v_full[vs], 32768);
            load_bf16_tile(slab ? &tm_cv : &tm_v, v_ptr(vs), key0, h, b, &v_full[vs]);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_s_bf16 = idesc_f32acc(1, 1, 0, 0, kAttnBM, kAttnBN);
      constexpr uint32_t idesc_s_f16 = idesc_f32acc(0, 0, 0, 0, kAttnBM, kAttnBN);
      constexpr uint32_t idesc_o_bf16 = idesc_f32acc(1, 1, 0, 1, kAttnBM, kAttnD);  // bf16 P, bf16 V
      constexpr uint32_t idesc_o16 = idesc_f32acc(0, 0, 0, 1, kAttnBM, kAttnD);     // f16 P, f16 V
      const uint32_t idesc_s = f16 ? idesc_s_f16 : idesc_s_bf16;
      const uint32_t idesc_o = f16 ? idesc_o16 : idesc_o_bf16;
      // S_g at column 128 g (P_g over its first 64 columns), O_g at 256 + 128 g
      bool ok = mbar_wait(q_full, 0, abort_flag, a.status);
      // Shared-memory descriptors of the Q tiles and of ring stage 0; another tile,
      // stage or K step is the same descriptor plus its byte offset / 16 (the 14-bit
      // address field never carries: every address is below 256 KB).  One 32 KB tile
      // or stage = 2048 in the field.  This keeps the single issuing thread to a few
      // instructions per MMA: it shares its sub-partition with four softmax warps.
      const uint64_t q_desc = sdesc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t k_desc = sdesc_sw128(smem_u32(k_ptr(0)), 16, 1024);
      const uint64_t v_desc = sdesc_sw128(smem_u32(v_ptr(0)), 16384, 1024);
      auto issue_s = [&](int g, int t) {  // K_t resident (k_full waited)
        const uint64_t qd0 = q_desc + static_cast<uint64_t>(g) * 2048u;
        const uint64_t kd0 = k_desc + static_cast<uint64_t>(t & 1) * 2048u;
#pragma unroll
        for (int k = 0; k < kAttnD / 16; ++k) {
          const uint32_t off16 = ((k >> 2) * 16384 + (k & 3) * 32) >> 4;
          umma_f16_ss(tmem + 128u * g, qd0 + off16, kd0 + off16, idesc_s, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[g]);
      };
      auto wait_k = [&](int t) -> bool {
        if (!mbar_wait(&k_full[t & 1], (t >> 1) & 1, abort_flag, a.status)) return false;
        tc_fence_after();
        return true;
      };
      auto issue_pv = [&](int g, int t) -> bool {
        const int vs = t & 1;
        if (!mbar_wait(&p_full[g], t & 1, abort_flag, a.status)) return false;
        if (g == 0 && !mbar_wait(&v_full[vs], (t >> 1) & 1, abort_flag, a.status)) return false;
        tc_fence_after();
        const uint64_t vd0 = v_desc + static_cast<uint64_t>(vs) * 2048u;
        const uint32_t idesc = (v_fp8 && t < n_slab) ? idesc_o16 : idesc_o;
#pragma unroll
        for (int k = 0; k < kAttnBN / 16; ++k) {
          // 16 keys per step: V rows [16k, 16k+16) (2048 B); d halves 16 KB apart
          // P of keys 16k .. 16k+15: 8 packed columns, keys 64-127 at S_g's columns 64-95
          const uint32_t p_col = 128u * g + k * 8 + (k >= kAttnBN / 32 ? 32u : 0u);
          umma_f16_ts(tmem + 256u + 128u * g, tmem + p_col, vd0 + k * 128u, idesc, (t > 0 || k > 0) ? 1u : 0u);
        }
        if (t == n_tiles - 1) umma_commit(&o_full[g]);
        if (g == kAttnTiles - 1) umma_commit(&v_empty[vs]);
        return true;
      };
      if (ok && wait_k(0)) {
        issue_s(0, 0);
        issue_s(1, 0);
        umma_commit(&k_empty[0]);
        for (int t = 0; t < n_tiles; ++t) {
          const bool next = t + 1 < n_tiles;
          if (!issue_pv(0, t)) break;
          if (next) {
            if (!wait_k(t + 1)) break;
            issue_s(0, t + 1);
          }
          if (!issue_pv(1, t)) break;
          if (next) {
            issue_s(1, t + 1);
            umma_commit(&k_empty[(t + 1) & 1]);
          }
        }
      }
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------ V converters
    if (v_fp8 && n_slab > 0) {
      const int ct = threadIdx.x - 64;  // 0..63
      for (int t = 0; t < n_slab; ++t) {
        const int s = t & 1;
        const uint32_t ph = (t >> 1) & 1;
        if (!mbar_wait(&v8_full[s], ph, abort_flag, a.status)) break;
        const uint8_t* raw = v8_ptr(s);
        uint8_t* dst = v_ptr(s);
        // 2048 chunks of 8 values: chunk g -> key row g / 16, d-chunk g % 16; the f16
        // tile is written in the 128-byte-swizzled layout TMA would produce.
        for (int g = ct; g < 2048; g += 64) {
          const int r = g >> 4, dc = g & 15;
          const uint2 w = *reinterpret_cast<const uint2*>(raw + r * 128 + dc * 8);
          const int hd = dc >> 3, c = dc & 7;
          *reinterpret_cast<uint4*>(dst + hd * 16384 + r * 128 + ((c ^ (r & 7)) << 4)) =
              make_uint4(cvt_e4m3x2_to_f16x2(static_cast<uint16_t>(w.x & 0xFFFFu)),
                         cvt_e4m3x2_to_f16x2(static_cast<uint16_t>(w.x >> 16)),
                         cvt_e4m3x2_to_f16x2(static_cast<uint16_t>(w.y & 0xFFFFu)),
                         cvt_e4m3x2_to_f16x2(static_cast<uint16_t>(w.y >> 16)));
        }
        fence_proxy_async_smem();
        named_bar_sync(1, 64);
        if (ct == 0) mbar_arrive(&v_full[s]);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax (tile g)
    // 8 warps per query tile; a warp covers 16 rows of its TMEM lane quarter with two
    // threads per row (16x32bx2 accesses): thread (row, hc) reads, masks and
    // exponentiates the scores of columns 64 hc .. 64 hc + 63, the row max is one
    // shuffle away (lane ^ 16), and the row sum is combined only at the end.
    const int sw = warp - 4;
    const int g = sw >> 3;
    const int quarter = sw & 3;      // TMEM lane quarter this warp may access (warp % 4)
    const int sub = (sw >> 2) & 1;   // its lower or upper 16 lanes
    const int hc = lane >> 4;        // column half of the row
    const int row = quarter * 32 + sub * 16 + (lane & 15);
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32 + sub * 16) << 16;
    const uint32_t tS = tmem + lane_base + 128u * g;  // S_g; P_g over the first half of each thread's scores
    const uint32_t tO = tmem + lane_base + 256u + 128u * g;
    const uint8_t* kvb = has_kv ? a.key_valid + static_cast<int64_t>(b) * a.kv_sb : nullptr;
    float m_run = -INFINITY, l_run = 0.0f;  // l_run: this thread's half of the row sum
    bool ok = true;
    // fp8 slab: the per-(b, h) V scale is applied to O once, after the last slab tile
    const bool slab_f16 = v_fp8 && n_slab > 0;
    const float vsc = slab_f16 ? __ldg(a.v_scale + static_cast<int64_t>(b) * a.H + h) : 1.0f;
    bool vsc_applied = !slab_f16;
    for (int t = 0; t < n_tiles; ++t) {
      // the warp leaves together (tcgen05.ld/st are warp-collective), also on a timeout
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[g], t & 1, abort_flag, a.status))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool slab = t < n_slab;
      const int kv0 = slab ? t * kAttnBN : P + (t - n_slab) * kAttnBN;
      const int seg_end = slab ? P : kv_total;
      // column c of the tile allowed iff c <= lim_rel (and key valid); this thread's
      // columns are 64 hc + j
      const int lim_rel = min(my_L, seg_end - 1) - kv0 - kAttnHalf * hc;
      // key-valid bits of this thread's columns: bit i of kvm[j] <-> column 64 hc + 32 j + i
      uint32_t kvm[2] = {0xffffffffu, 0xffffffffu};
      if (has_kv) {
        uint32_t all[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int kv = kv0 + 32 * j + lane;
          const bool valid = kv < seg_end && __ldg(kvb + kv) != 0;
          all[j] = __ballot_sync(0xffffffffu, valid);
        }
        kvm[0] = hc ? all[2] : all[0];
        kvm[1] = hc ? all[3] : all[1];
      }
      float sv[kAttnHalf];
      {
        uint32_t r[kAttnHalf];
        tmem_ld_2x64(tS, r);
#pragma unroll
        for (int j = 0; j < kAttnHalf; ++j) sv[j] = __uint_as_float(r[j]);
      }
      // raw scores stay unscaled; the scale is folded into the exponent below
      // every key of the tile allowed for every row of the warp (warp-uniform: the
      // branches below end in warp-collective TMEM stores)
      const bool full = __all_sync(0xffffffffu, lim_rel + kAttnHalf * hc >= kAttnBN - 1 && !has_kv);
      float mx[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) mx[i] = -INFINITY;
      if (full) {
#pragma unroll
        for (int c = 0; c < kAttnHalf; c += 8) {
          mx[0] = fmax3(mx[0], sv[c], sv[c + 1]);
          mx[1] = fmax3(mx[1], sv[c + 2], sv[c + 3]);
          mx[2] = fmax3(mx[2], sv[c + 4], sv[c + 5]);
          mx[3] = fmax3(mx[3], sv[c + 6], sv[c + 7]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < kAttnHalf; ++c) {
          const bool allowed = (c <= lim_rel) && ((kvm[c >> 5] >> (c & 31)) & 1u);
          sv[c] = allowed ? sv[c] : -INFINITY;
          mx[c & 3] = fmaxf(mx[c & 3], sv[c]);
        }
      }
      float raw_max = fmax3(mx[0], mx[1], fmaxf(mx[2], mx[3]));
      raw_max = fmaxf(raw_max, __shfl_xor_sync(0xffffffffu, raw_max, 16));  // the row's other half
      const float tmax = raw_max * a.qk_scale_log2;  // scale > 0: max commutes with it
      // the running max moves (and O, l are rescaled) only when it grows by > 2^8; both
      // threads of a row see the same values and decide alike
      float alpha = 1.0f;
      bool rescale_o = false;
      if (tmax > m_run + kRescaleThreshold || (m_run == -INFINITY && tmax > -INFINITY)) {
        alpha = (m_run == -INFINITY) ? 0.0f : ex2(m_run - tmax);
        rescale_o = (m_run != -INFINITY);
        m_run = tmax;
      }
      const float neg_m = (m_run == -INFINITY) ? 0.0f : -m_run;
      // S_g(t) is in registers: P_g(t) overwrites the first 32 of each thread's columns
      const bool f16p = f16 || (slab_f16 && slab);
      float psum;
      if (full)
        psum = f16p ? softmax_half_row<true, true>(sv, a.qk_scale_log2, neg_m, tS)
                    : softmax_half_row<true, false>(sv, a.qk_scale_log2, neg_m, tS);
      else
        psum = f16p ? softmax_half_row<false, true>(sv, a.qk_scale_log2, neg_m, tS)
                    : softmax_half_row<false, false>(sv, a.qk_scale_log2, neg_m, tS);
      l_run = l_run * alpha + psum;
      // O_g holds the sum up to tile t-1 (P_g(t-1).V completed before S_g(t)): it is
      // touched only when some row of the warp rescales (or at the slab boundary);
      // the whole warp then runs the warp-collective TMEM loads/stores, a row that
      // keeps its max with factor 1.
      const bool boundary = !vsc_applied && t == n_slab;  // first fresh tile after the fp8 slab
      if (t >= 1 && __any_sync(0xffffffffu, rescale_o || boundary)) {
        const float f = (rescale_o ? alpha : 1.0f) * (boundary ? vsc : 1.0f);
#pragma unroll
        for (int c = 0; c < kAttnHalf / 32; ++c) {
          uint32_t r[32];
          tmem_ld_2x32(tO + c * 32, r);
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * f);
          tmem_st_2x32(tO + c * 32, r);
        }
        if (boundary) vsc_applied = true;
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[g]);
    }
    // epilogue: O / l -> bf16, each thread its row's half (columns 64 hc ..)
    const float l_row = l_run + __shfl_xor_sync(0xffffffffu, l_run, 16);
    const int grow = m0 + g * kAttnBM + row;
    float o[kAttnHalf];
    bool have_o = false;
    const bool o_ready = ok && n_tiles > 0 && mbar_wait(&o_full[g], 0, abort_flag, a.status);
    if (__all_sync(0xffffffffu, o_ready)) {  // warp-uniform: tcgen05.ld is warp-collective
      tc_fence_after();
      uint32_t r[kAttnHalf];
      tmem_ld_2x64(tO, r);
#pragma unroll
      for (int j = 0; j < kAttnHalf; ++j) o[j] = __uint_as_float(r[j]);
      have_o = true;
    }
    uint32_t am2 = 0;  // two running bf16 |out| maxima (amax_out)
    if (grow < a.SQ) {
      const bool nz = have_o && l_row > 0.0f;
      const float inv = nz ? (vsc_applied ? 1.0f : vsc) / l_row : 0.0f;
      uint16_t* dst = a.out + static_cast<int64_t>(b) * a.o_sb + static_cast<int64_t>(grow) * a.o_ss +
                      static_cast<int64_t>(h) * a.o_sh + kAttnHalf * hc;
#pragma unroll
      for (int c = 0; c < kAttnHalf; c += 8) {
        uint4 w = make_uint4(0u, 0u, 0u, 0u);
        if (nz && f16)
          w = make_uint4(pack_f16x2(o[c] * inv, o[c + 1] * inv), pack_f16x2(o[c + 2] * inv, o[c + 3] * inv),
                         pack_f16x2(o[c + 4] * inv, o[c + 5] * inv), pack_f16x2(o[c + 6] * inv, o[c + 7] * inv));
        else if (nz)
          w = make_uint4(pack_bf16x2(o[c] * inv, o[c + 1] * inv), pack_bf16x2(o[c + 2] * inv, o[c + 3] * inv),
                         pack_bf16x2(o[c + 4] * inv, o[c + 5] * inv), pack_bf16x2(o[c + 6] * inv, o[c + 7] * inv));
        am2 = __vmaxu2(am2, __vmaxu2(__vmaxu2(w.x & 0x7FFF7FFFu, w.y & 0x7FFF7FFFu),
                                     __vmaxu2(w.z & 0x7FFF7FFFu, w.w & 0x7FFF7FFFu)));
        *reinterpret_cast<uint4*>(dst + c) = w;
      }
    }
    if (a.amax_out) {  // CTA-uniform: the whole warp reduces
      // |out| bit patterns order like the values for either 16-bit type; the largest one
      // is widened to fp32 bits (bf16: the top half; fp16: an exact conversion)
      const uint32_t m = __reduce_max_sync(0xffffffffu, max(am2 & 0xFFFFu, am2 >> 16));
      const uint32_t bits =
          f16 ? __float_as_uint(__half2float(__ushort_as_half(static_cast<unsigned short>(m)))) : m << 16;
      if (lane == 0 && m != 0u) atomicMax(a.amax_out, bits);
    }
  }

  tc_fence_before();
  __syncthreads();
  pdl_trigger();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// 4-D map (d, s, h, b) over a [B, S, H, D] tensor with element strides (sb, ss, sh).
static int make_bshd_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int esize, int64_t B, int64_t S,
                         int64_t H, int64_t sb, int64_t ss, int64_t sh, uint32_t box_d, CUtensorMapSwizzle sw) {
  const uint64_t dims[4] = {static_cast<uint64_t>(kAttnD), static_cast<uint64_t>(S), static_cast<uint64_t>(H),
                            static_cast<uint64_t>(B)};
  const uint64_t strides[3] = {static_cast<uint64_t>(ss * esize), static_cast<uint64_t>(sh * esize),
                               static_cast<uint64_t>(sb * esize)};
  const uint32_t box[4] = {box_d, static_cast<uint32_t>(kAttnBN), 1, 1};
  return make_tmap_nd(m, base, dt, 4, dims, strides, box, sw);
}

}  // namespace qik

using namespace qik;

extern "C" int qik_block_causal_attention(const qik_attn_args* args, int* status, void* stream) {
  QIK_REQUIRE(args != nullptr, "qik_block_causal_attention: args is NULL");
  const qik_attn_args& A = *args;
  QIK_REQUIRE(A.D == kAttnD, "qik_block_causal_attention: head_dim %lld unsupported (128 only)", (long long)A.D);
  QIK_REQUIRE(A.B >= 0 && A.SQ >= 0 && A.SN >= 0 && A.P >= 0 && A.H > 0, "qik_block_causal_attention: bad sizes");
  if (A.B == 0 || A.SQ == 0) return QIK_OK;
  QIK_REQUIRE(A.B * A.H <= 65535 && (A.SQ + kAttnRows - 1) / kAttnRows <= 65535 && A.SN + A.P <= (1ll << 30),
              "qik_block_causal_attention: size out of range");
  // SN == 0: the rows attend to the cache alone (or, without one, to no key: zeros);
  // k and v are then never read and may be empty
  const bool fresh = A.SN > 0;
  QIK_REQUIRE(A.q && A.out && (!fresh || (A.k && A.v)), "qik_block_causal_attention: NULL q/k/v/out");
  const bool has_cache = (A.flags & QIK_ATTN_HAS_CACHE) && A.P > 0;
  const bool v_fp8 = has_cache && (A.flags & QIK_ATTN_V_FP8);
  QIK_REQUIRE(!has_cache || (A.cache_k && A.cache_v), "qik_block_causal_attention: cache pointers missing");
  QIK_REQUIRE(!v_fp8 || A.cache_v_scale, "qik_block_causal_attention: fp8 V needs cache_v_scale");
  QIK_REQUIRE((A.flags & QIK_ATTN_UNIFORM) || A.L, "qik_block_causal_attention: L is NULL");
  QIK_REQUIRE(!(A.flags & QIK_ATTN_HAS_KEY_VALID) || A.key_valid, "qik_block_causal_attention: key_valid is NULL");
  auto ok_strides = [](int64_t sb, int64_t ss, int64_t sh, int esize) {
    return (sb * esize) % 16 == 0 && (ss * esize) % 16 == 0 && (sh * esize) % 16 == 0 && sb >= 0 && ss > 0 && sh > 0;
  };
  QIK_REQUIRE(ok_strides(A.q_sb, A.q_ss, A.q_sh, 2) && ok_strides(A.o_sb, A.o_ss, A.o_sh, 2) &&
                  (!fresh || (ok_strides(A.k_sb, A.k_ss, A.k_sh, 2) && ok_strides(A.v_sb, A.v_ss, A.v_sh, 2))),
              "qik_block_causal_attention: q/k/v/out strides must be multiples of 16 bytes (unit stride on D)");
  QIK_REQUIRE(aligned16(A.q) && aligned16(A.out) && (!fresh || (aligned16(A.k) && aligned16(A.v))),
              "qik_block_causal_attention: q/k/v/out must be 16-byte aligned");
  if (has_cache) {
    QIK_REQUIRE(ok_strides(A.ck_sb, A.ck_ss, A.ck_sh, 2) && ok_strides(A.cv_sb, A.cv_ss, A.cv_sh, v_fp8 ? 1 : 2) &&
                    aligned16(A.cache_k) && aligned16(A.cache_v),
                "qik_block_causal_attention: cache strides/alignment must be 16-byte multiples");
  }
  CUtensorMap tq, tk, tv, tck, tcv;
  const CUtensorMapDataType dt16 =
      (A.flags & QIK_ATTN_F16) ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  int rc = make_bshd_map(&tq, A.q, dt16, 2, A.B, A.SQ, A.H, A.q_sb, A.q_ss, A.q_sh, 64,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc && fresh)
    rc = make_bshd_map(&tk, A.k, dt16, 2, A.B, A.SN, A.H, A.k_sb, A.k_ss, A.k_sh, 64,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc && fresh)
    rc = make_bshd_map(&tv, A.v, dt16, 2, A.B, A.SN, A.H, A.v_sb, A.v_ss, A.v_sh, 64,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (!fresh) tk = tv = tq;  // never read: no fresh key tile exists
  if (has_cache) {
    rc = make_bshd_map(&tck, A.cache_k, dt16, 2, A.B, A.P, A.H, A.ck_sb, A.ck_ss, A.ck_sh,
                       64, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc) {
      if (v_fp8)
        rc = make_bshd_map(&tcv, A.cache_v, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, A.B, A.P, A.H, A.cv_sb, A.cv_ss,
                           A.cv_sh, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
      else
        rc = make_bshd_map(&tcv, A.cache_v, dt16, 2, A.B, A.P, A.H, A.cv_sb, A.cv_ss,
                           A.cv_sh, 64, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (rc) return rc;
  } else {
    tck = tk;
    tcv = tv;
  }
  AttnDev d;
  d.L = A.L;
  d.key_valid = A.key_valid;
  d.v_scale = A.cache_v_scale;
  d.out = static_cast<uint16_t*>(A.out);
  d.o_sb = A.o_sb;
  d.o_ss = A.o_ss;
  d.o_sh = A.o_sh;
  d.kv_sb = A.kv_sb;
  d.SQ = static_cast<int>(A.SQ);
  d.SN = static_cast<int>(A.SN);
  d.P = static_cast<int>(A.P);
  d.H = static_cast<int>(A.H);
  d.qk_scale_log2 = A.sm_scale * 1.4426950408889634f;
  d.flags = A.flags;
  d.status = status;
  d.amax_out = A.amax_out;
  static std::once_flag attr_once[64];
  int dev = 0;
  QIK_TRY_CUDA(cudaGetDevice(&dev));
  QIK_REQUIRE(dev >= 0 && dev < 64, "qik_block_causal_attention: device ordinal %d out of range", dev);
  cudaError_t attr_rc = cudaSuccess;
  std::call_once(attr_once[dev], [&] {
    attr_rc = cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnSmem::kBytes);
  });
  QIK_TRY_CUDA(attr_rc);
  // x = (b, h), y = query block (numbered from the last block: heaviest first)
  dim3 grid(static_cast<unsigned>(A.B * A.H), static_cast<unsigned>((A.SQ + kAttnRows - 1) / kAttnRows));
  // a programmatic dependent of the previous kernel in the stream (its prologue overlaps
  // that kernel's tail; the kernel waits for it before reading any input)
  QIK_TRY_CUDA(launch_kernel(attn_fwd_kernel, grid, dim3(kAttnThreads), AttnSmem::kBytes,
                             static_cast<cudaStream_t>(stream), true, tq, tk, tv, tck, tcv, d));
  return check_launch("attn_fwd_kernel");
}
