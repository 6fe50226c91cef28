// K5 — grouped expert GEMM on the 5th-generation tensor cores (sm_100a), single-CTA tiles.
//
// One persistent kernel computes C[g] = epilogue(A[rows of group g] . B[weight(g)]^T) for every
// row group g of up to two segments (segment 0: routed experts with device-side row offsets;
// segment 1: the shared expert over all tokens).  It replaces the per-expert loop
// tokens[idx] = expert(tokens[idx]) (src/qosmoe/async_cpu.py:137-173,
// src/qosmoe/moe_layer.py:226-253, qwen_ep_adapter/qwen_ep.py:85-89) and the shared expert
// (qwen_ep.py:94).  This file holds the 128-row tile form (tile_rows = 128); the default
// 256-row CTA-pair form is in gemm_sm100_pair.cu.
//
// Tile: 128 (token rows) x 256 (weight rows) x 64 (K) per stage, bf16 in, fp32 accumulate in TMEM.
//   warp 0      TMA producer (one thread): A 128x64 and B 256x64 tiles, 128-byte swizzle,
//               4-stage ring guarded by full/empty mbarriers.  No multicast.
//   warp 1      TMEM allocator (512 columns = two 128x256 fp32 accumulators) and MMA issuer
//               (one thread): 4 x tcgen05.mma (M128 N256 K16) per stage, tcgen05.commit frees
//               the stage and, after the last K block, signals the accumulator full.
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns, activation, bf16 pack, masked
//               16-byte stores; the accumulator is released as soon as it has been read, so
//               the next tile's MMAs overlap this tile's stores.
// SwiGLU weights are packed in 256-row blocks of 128 gate rows then the 128 matching up rows, so
// one 256-column accumulator row yields 128 finished SiLU(g) * u channels.
// Tiles follow the boustrophedon schedule of gemm_sm100.cuh (the longer-K segment first,
// group-major inside a segment).  Group row offsets are read on the device, so no host sync is
// needed.
// Every wait is bounded (2 s): on a timeout the kernel records DSCA_ERR_WAIT_TIMEOUT in the
// error word, drains its own outstanding copies and MMAs, frees TMEM and returns.
#include <algorithm>

#include "gemm_sm100.cuh"

namespace dsca {
namespace gemm {

constexpr int BM = 128;

// Stage layout.  bf16: A 128 x 64 and B 256 x 64, 4 stages.  F8 (fp8-e4m3 weights, the tokens as
// two e4m3 planes, fp8_split.cuh): 128 bytes of K per row as in bf16 — 128 elements — with the
// A tile's hi and lo planes, two tcgen05.mma.kind::f8f6f4 per 32-byte K step into the same
// accumulator (the bf16 MMA's tensor time per K element, half its weight bytes), 3 stages.
template <bool F8>
struct SCfg {
  static constexpr int kStages = F8 ? 3 : 4;
  static constexpr int kKE = F8 ? 128 : BK;         // K elements per stage
  static constexpr int kAPlane = BM * 128;          // 16 KB
  static constexpr int kABytes = (F8 ? 2 : 1) * kAPlane;
  static constexpr int kBBytes = BN * 128;          // 32 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024;  // + alignment slack
};

// D(tmem) (+)= A(smem desc) * B(smem desc), e4m3 x e4m3, fp32 accumulate
__device__ __forceinline__ void umma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

template <int EPI, bool F8>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmB0,
                        const __grid_constant__ CUtensorMap tmA1, const __grid_constant__ CUtensorMap tmB1,
                        const Params p) {
  using C = SCfg<F8>;
  constexpr int kStages = C::kStages, kABytes = C::kABytes, kBBytes = C::kBBytes, kStageBytes = C::kStageBytes;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ SmemCtl ctl;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t smem_a = smem_u32(smem);
  const uint32_t smem_b = smem_a + kStages * kABytes;

  const int warp = warp_id(), lane = lane_id();
  volatile int* abort_flag = &ctl.abort_flag;
  pdl_launch_dependents();  // a programmatic dependent (GEMM2) may be scheduled as SMs free up

  // ---- prologue: barriers, TMEM, group tile table
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&ctl.full[s]), 1);
      mbar_init(smem_u32(&ctl.empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&ctl.tmem_full[a]), 1);
      mbar_init(smem_u32(&ctl.tmem_empty[a]), 128);
    }
    for (int i = 0; i < kTQ; ++i) {
      mbar_init(smem_u32(&ctl.tq_full[i]), 1);
      mbar_init(smem_u32(&ctl.tq_empty[i]), 5);  // the MMA thread and the four epilogue warps
    }
    mbar_init(smem_u32(&ctl.mma_done), 1);
    ctl.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA0);
    prefetch_tmap(&tmB0);
    if (p.nseg > 1) {
      prefetch_tmap(&tmA1);
      prefetch_tmap(&tmB1);
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctl.tmem_base), kTmemCols);
    tmem_relinquish();
  }
  if (warp == 2) build_group_table<BM>(p, ctl, lane);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctl.tmem_base;
  const int total = ctl.total_tiles;

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int pending_phase[kStages];
      for (int i = 0; i < kStages; ++i) pending_phase[i] = -1;
      bool ok = true;
      bool seg0_ready = !p.pdl_seg0_wait;
      const uint64_t pol_first = l2_policy_evict_first(), pol_last = l2_policy_evict_last();
      // the tile of round r: drawn (static or ticket) and published to the MMA and epilogue
      // warps; -1 past the last tile, -2 when the wait for a free queue slot gave up
      auto publish = [&](int r) -> int {
        const int slot = r % kTQ;
        if (!mbar_wait(smem_u32(&ctl.tq_empty[slot]), (uint32_t)(((r / kTQ) & 1) ^ 1), abort_flag, p.err))
          return -2;
        int tile = ticket_tile(p, r, (int)blockIdx.x, (int)gridDim.x);
        if (tile >= total) tile = -1;
        *reinterpret_cast<volatile int*>(&ctl.tq[slot]) = tile;
        mbar_arrive(smem_u32(&ctl.tq_full[slot]));
        return tile;
      };
      int next = publish(0);
      for (int r = 0; ok; ++r) {
        if (next == -2) {
          ok = false;
          break;
        }
        const int tile = next;
        if (tile < 0) break;
        // the next round's tile is drawn one tile ahead: the ticket's latency overlaps this
        // tile's loads instead of delaying the next tile's first stage
        next = publish(r + 1);
        const TileInfo ti = decode<BM>(p, ctl, tile);
        const CUtensorMap* ma = ti.seg == 0 ? &tmA0 : &tmA1;
        const CUtensorMap* mb = ti.seg == 0 ? &tmB0 : &tmB1;
        if (ti.seg == 0 && !seg0_ready) {
          pdl_wait();  // the preceding kernel (the permute) has written the rows
          seg0_ready = true;
        }
        const int kb_n = p.seg[ti.seg].k_blocks;
        // routed tile: L2 prefetch of the boxes beyond the shared-memory stages, then one box
        // l2_ahead K blocks ahead of every load
        const int pf = ti.seg == 0 ? p.l2_ahead : 0;
        for (int kb = kStages; kb < min(pf, kb_n); ++kb) {
          tma_prefetch_l2_2d(mb, kb * C::kKE, ti.b_row0);
          tma_prefetch_l2_2d(ma, kb * C::kKE, ti.row0);
        }
        for (int kb = 0; kb < kb_n; ++kb) {
          if (!mbar_wait(smem_u32(&ctl.empty[s]), ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
          const uint32_t fb = smem_u32(&ctl.full[s]);
          mbar_arrive_expect_tx(fb, kStageBytes);
          const int kx = kb * C::kKE;
          if (pf > 0 && kb + pf < kb_n && kb + pf >= kStages) {
            tma_prefetch_l2_2d(mb, (kb + pf) * C::kKE, ti.b_row0);
            tma_prefetch_l2_2d(ma, (kb + pf) * C::kKE, ti.row0);
          }
          if (p.l2_hints) {
            tma_load_2d_hint(smem_a + s * kABytes, ma, fb, kx, ti.row0, pol_last);
            if constexpr (F8)  // the lo plane of the same token rows
              tma_load_2d_hint(smem_a + s * kABytes + C::kAPlane, ma, fb, p.seg[ti.seg].t_lo + kx, ti.row0, pol_last);
            tma_load_2d_hint(smem_b + s * kBBytes, mb, fb, kx, ti.b_row0, ti.seg == 0 ? pol_first : pol_last);
          } else {
            tma_load_2d(smem_a + s * kABytes, ma, fb, kx, ti.row0);
            if constexpr (F8) tma_load_2d(smem_a + s * kABytes + C::kAPlane, ma, fb, p.seg[ti.seg].t_lo + kx, ti.row0);
            tma_load_2d(smem_b + s * kBBytes, mb, fb, kx, ti.b_row0);
          }
          pending_phase[s] = (int)ph;
          if (++s == kStages) { s = 0; ph ^= 1u; }
        }
      }
      if (!ok) {
        // drain: the last issued load of every stage must land before the CTA exits
        for (int i = 0; i < kStages; ++i)
          if (pending_phase[i] >= 0) mbar_drain(smem_u32(&ctl.full[i]), (uint32_t)pending_phase[i]);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = F8 ? idesc_e4m3_f32(BM, BN) : idesc_bf16_f32(BM, BN);
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      bool ok = true;
      for (int r = 0; ok; ++r, ++it) {
        const int tile = tq_take<false>(ctl, r, abort_flag, p.err, nullptr);
        if (tile < 0) {
          ok = *abort_flag == 0;
          break;
        }
        const TileInfo ti = decode<BM>(p, ctl, tile);
        const int acc = it & 1;
        const uint32_t acc_ph = (uint32_t)((it >> 1) & 1);
        if (!mbar_wait(smem_u32(&ctl.tmem_empty[acc]), acc_ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        const int kb_n = p.seg[ti.seg].k_blocks;
        for (int kb = 0; kb < kb_n; ++kb) {
          if (!mbar_wait(smem_u32(&ctl.full[s]), ph, abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = sw128_kmajor_desc(smem_a + s * kABytes);
          const uint64_t bdesc = sw128_kmajor_desc(smem_b + s * kBBytes);
          if constexpr (F8) {
            const uint64_t ldesc = sw128_kmajor_desc(smem_a + s * kABytes + C::kAPlane);
#pragma unroll
            for (int k = 0; k < C::kKE / 32; ++k) {
              const uint64_t ko = (uint64_t)(2 * k);
              umma_f8(d_tmem, adesc + ko, bdesc + ko, idesc, (kb > 0 || k > 0) ? 1u : 0u);
              umma_f8(d_tmem, ldesc + ko, bdesc + ko, idesc, 1u);
            }
          } else {
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              umma_f16(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc,
                       (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(smem_u32(&ctl.empty[s]));
          if (++s == kStages) { s = 0; ph ^= 1u; }
        }
        if (!ok) break;
        umma_commit(smem_u32(&ctl.tmem_full[acc]));
      }
      if (!ok) {
        // aborting: wait until every MMA this thread issued has completed before TMEM is freed
        umma_commit(smem_u32(&ctl.mma_done));
        mbar_drain(smem_u32(&ctl.mma_done), 0);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5 -> TMEM lane quarters 2, 3, 0, 1)
    const int q = warp & 3;
    const int r_in_tile = q * 32 + lane;
    int it = 0;
    for (int r = 0;; ++r, ++it) {
      int tile = 0;
      if (lane == 0) tile = tq_take<false>(ctl, r, abort_flag, p.err, nullptr);
      tile = __shfl_sync(0xffffffffu, tile, 0);
      if (tile < 0) break;
      const TileInfo ti = decode<BM>(p, ctl, tile);
      const Segment& sg = p.seg[ti.seg];
      const int acc = it & 1;
      const uint32_t acc_ph = (uint32_t)((it >> 1) & 1);
      // one lane polls, the warp follows its verdict (tcgen05.ld below must not diverge)
      int ok = 1;
      if (lane == 0) ok = mbar_wait(smem_u32(&ctl.tmem_full[acc]), acc_ph, abort_flag, p.err) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      bool valid = r_in_tile < ti.rows_valid;
      const size_t row = (size_t)(ti.row0 + r_in_tile);
      __nv_bfloat16* crow = sg.c + row * (size_t)sg.ldc;
      if (EPI == kEpiStore && sg.ep != nullptr && valid) {
        // expert parallel: this row goes back to the rank that sent it (NVLink store)
        crow = ep_return_row(sg.ep, ti.group, (int)row, sg.ldc);
        if (crow == nullptr) {
          record_error(p.err, kErrIndex);
          valid = false;
        }
      }
      // F8: this row's 1 / s (the token scale); the weight row scales are per column below
      const float ts = (F8 && valid) ? __ldg(sg.t_scale + row) : 0.0f;
      if constexpr (EPI == kEpiSwiGLU) {
        const int col0 = ti.n_blk * (BN / 2);
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
          // accumulator columns: 128 gate channels, then the 128 matching up channels
          uint32_t g[32], u[32];
          tmem_ld32(taddr + c, g);
          tmem_ld32(taddr + BN / 2 + c, u);
          tmem_wait_ld();
          if constexpr (F8) {
            // weight rows b_row0 + c + i (gate) and b_row0 + 128 + c + i (up) (packed rows past a
            // group's channels are zero)
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              g[i] = __float_as_uint(__uint_as_float(g[i]) * __ldg(sg.w_scale + ti.b_row0 + c + i) * ts);
              u[i] = __float_as_uint(__uint_as_float(u[i]) * __ldg(sg.w_scale + ti.b_row0 + BN / 2 + c + i) * ts);
            }
          }
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float g0 = __uint_as_float(g[2 * i]), g1 = __uint_as_float(g[2 * i + 1]);
            float u0 = __uint_as_float(u[2 * i]), u1 = __uint_as_float(u[2 * i + 1]);
            packed[i] = pack_bf16x2(silu(g0) * u0, silu(g1) * u1);
          }
          const int col = col0 + c;
          if (valid && col < sg.n_store) {
            uint4* dst = reinterpret_cast<uint4*>(crow + col);
#pragma unroll
            for (int v = 0; v < 4; ++v)
              if (col + v * 8 < sg.n_store)
                dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
          }
        }
      } else {
        const int col0 = ti.n_blk * BN;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t v32[32];
          tmem_ld32(taddr + c, v32);
          tmem_wait_ld();
          if constexpr (F8) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              v32[i] = __float_as_uint(__uint_as_float(v32[i]) * __ldg(sg.w_scale + ti.b_row0 + c + i) * ts);
          }
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float a0 = __uint_as_float(v32[2 * i]), a1 = __uint_as_float(v32[2 * i + 1]);
            if constexpr (EPI == kEpiReLU) {
              a0 = fmaxf(a0, 0.0f);
              a1 = fmaxf(a1, 0.0f);
            }
            packed[i] = pack_bf16x2(a0, a1);
          }
          const int col = col0 + c;
          if (valid && col < sg.n_store) {
            uint4* dst = reinterpret_cast<uint4*>(crow + col);
#pragma unroll
            for (int v = 0; v < 4; ++v)
              if (col + v * 8 < sg.n_store)
                dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&ctl.tmem_empty[acc]));
      if (p.seg1_done != nullptr && ti.seg == 1) seg1_tile_stored(p, ctl, lane, 4u);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0) tile_counter_exit(p);
  if (p.ep_signal != nullptr) ep::signal_when_grid_done(p.ep_signal, &p.ep_signal->return_done, ep::kReturn);
}

}  // namespace gemm

// ------------------------------------------------------------------ host side
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    fn = reinterpret_cast<PFN_encodeTiled>(ptr);
  }
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix, box = box_rows x 64, 128B swizzle.
int make_map_bf16(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  PFN_encodeTiled enc = get_encode_fn();
  if (enc == nullptr) return DSCA_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (cols * 2) % 16 != 0) return DSCA_ERR_BAD_ARG;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DSCA_OK : DSCA_ERR_CUDA;
}

template <int EPI, bool F8 = false>
static int launch_kernel(const CUtensorMap& a0, const CUtensorMap& b0, const CUtensorMap& a1, const CUtensorMap& b1,
                         const gemm::Params& p, int grid, cudaStream_t stream) {
  static PerDeviceOnce attr_once;
  auto kern = gemm::grouped_gemm_kernel<EPI, F8>;
  constexpr int smem_bytes = gemm::SCfg<F8>::kSmemBytes;
  if (attr_once.run([&] {
        return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
      }) != cudaSuccess)
    return DSCA_ERR_CUDA;
  if (!p.pdl_seg0_wait) {
    kern<<<grid, gemm::kThreads, smem_bytes, stream>>>(a0, b0, a1, b1, p);
    return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
  }
  // programmatic dependent of the permute: may start while it runs (see Params::pdl_seg0_wait)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(gemm::kThreads);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, a0, b0, a1, b1, p) != cudaSuccess) return DSCA_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

static int launch_one(int epi, const CUtensorMap& a0, const CUtensorMap& b0, const CUtensorMap& a1,
                      const CUtensorMap& b1, const gemm::Params& p, int grid, cudaStream_t stream) {
  switch (epi) {
    case gemm::kEpiSwiGLU: return launch_kernel<gemm::kEpiSwiGLU>(a0, b0, a1, b1, p, grid, stream);
    case gemm::kEpiReLU: return launch_kernel<gemm::kEpiReLU>(a0, b0, a1, b1, p, grid, stream);
    default: return launch_kernel<gemm::kEpiStore>(a0, b0, a1, b1, p, grid, stream);
  }
}

int launch_grouped_ffn_bf16(const dsca_ffn_args* f, int num_sms, cudaStream_t stream) {
  const int phases_all = f->phases == 0 ? 3 : f->phases;
  if (f->tile_rows == 256 || f->tile_rows == 512) return launch_grouped_ffn_bf16_pair(f, num_sms, stream);
  if (f->tile_rows == 0) {
    // default: the CTA-pair swap-AB kernel for GEMM2 and a ReLU GEMM1.  A SwiGLU GEMM1 with both
    // segments in this call and 4096 or more tokens takes the pair kernel too (the gate and up
    // rows of a CTA's 64 channels as one operand: measured faster there), otherwise single-CTA
    // 128-token tiles (more tiles for fewer tokens: faster at 1024 tokens)
    const bool glu = f->act == DSCA_ACT_SWIGLU;
    dsca_ffn_args g = *f;
    int rc;
    // shared-expert handoff between the two launches (see dsca_ffn_args::shared_handoff); 2
    // marks it as arranged here for the two launches below
    const int segs = f->segments == 0 ? 3 : f->segments;
    const bool handoff = f->shared_handoff == 1 && glu && phases_all == 3 && f->tile_counters != nullptr &&
                         f->pdl_after_permute && f->ep_ctx == nullptr && f->shared_rows > 0 && segs == 3;
    g.shared_handoff = handoff ? 2 : 0;
    const int rows1 = f->shared_rows > 0 ? f->shared_rows : f->capacity;
    const bool pair1 = glu && segs == 3 && rows1 >= 4096;
    if (phases_all & 1) {
      g.phases = 1;
      g.tile_rows = (pair1 || !glu) ? 256 : 128;
      if ((rc = launch_grouped_ffn_bf16(&g, num_sms, stream))) return rc;
    }
    if (phases_all & 2) {
      g.phases = 2;
      g.tile_rows = 256;
      if ((rc = launch_grouped_ffn_bf16(&g, num_sms, stream))) return rc;
    }
    return DSCA_OK;
  }
  const int grid = f->num_ctas > 0 ? f->num_ctas : num_sms;
  const int segs = f->segments == 0 ? 3 : f->segments;
  const bool shared = f->shared_rows > 0 && (segs & 2);
  const bool routed = (segs & 1) != 0;
  const int phases = phases_all;
  if (!routed && !shared) return DSCA_OK;
  int rc;
  // ---- GEMM1: h = act(a . w1^T)   (+ hs = act(xs . ws1^T))
  if (phases & 1) {
    CUtensorMap a0, b0, a1, b1;
    if ((rc = make_map_bf16(&a0, f->a, (uint64_t)f->capacity, (uint64_t)f->d, gemm::BM))) return rc;
    if ((rc = make_map_bf16(&b0, f->w1, (uint64_t)f->num_experts_w * f->n1p, (uint64_t)f->d, gemm::BN))) return rc;
    if (shared) {
      if ((rc = make_map_bf16(&a1, f->xs, (uint64_t)f->shared_rows, (uint64_t)f->d, gemm::BM))) return rc;
      if ((rc = make_map_bf16(&b1, f->ws1, (uint64_t)f->shared_n1p, (uint64_t)f->d, gemm::BN))) return rc;
    } else {
      a1 = a0;
      b1 = b0;
    }
    gemm::Params p{};
    const int epi = f->act == DSCA_ACT_SWIGLU ? gemm::kEpiSwiGLU : gemm::kEpiReLU;
    p.epi = epi;
    p.tile_counter = f->tile_counters;  // GEMM1: [0, 2)
    p.seg1_done = (f->shared_handoff == 2 && shared) ? f->tile_counters + 4 : nullptr;  // [4, 6)
    p.err = f->err;
    p.nseg = shared ? 2 : 1;
    // equal K (the model width) in both segments; after a permute launched just before, the
    // shared-expert tiles go first so that they overlap it (programmatic dependent launch)
    p.pdl_seg0_wait = (f->pdl_after_permute && routed) ? 1 : 0;
    p.seg_first = (p.pdl_seg0_wait && shared) ? 1 : 0;
    // interleaved segments: two rounds of shared tiles first when the permute is still running
    p.l2_hints = f->cache_hints & 1;
    p.l2_ahead = (f->cache_hints >> 8) & 0xff;
    p.interleave_lead = (shared && routed && (f->tile_order & 1)) ? (p.pdl_seg0_wait ? 2 * grid : 0) : -1;
    gemm::set_weight_major(p, f->tile_order);
    gemm::Segment& s0 = p.seg[0];
    s0.group_offsets = f->group_offsets;
    s0.group_weight = f->group_weight;
    s0.group_order = f->group_order;
    s0.ngroups = routed ? f->num_groups : 0;
    s0.rows = 0;
    s0.n_tiles = f->n1p / gemm::BN;
    s0.b_rows_per_group = f->n1p;
    s0.k_blocks = (f->d + gemm::BK - 1) / gemm::BK;
    s0.c = reinterpret_cast<__nv_bfloat16*>(f->h);
    s0.ldc = f->ip;
    s0.n_store = f->ip;
    s0.capacity = f->capacity;
    if (shared) {
      gemm::Segment& s1 = p.seg[1];
      s1.group_offsets = nullptr;
      s1.group_weight = nullptr;
      s1.ngroups = 1;
      s1.rows = f->shared_rows;
      s1.n_tiles = f->shared_n1p / gemm::BN;
      s1.b_rows_per_group = f->shared_n1p;
      s1.k_blocks = (f->d + gemm::BK - 1) / gemm::BK;
      s1.c = reinterpret_cast<__nv_bfloat16*>(f->hs);
      s1.ldc = f->shared_ip;
      s1.n_store = f->shared_ip;
      s1.capacity = f->shared_rows;
    }
    if ((rc = launch_one(epi, a0, b0, a1, b1, p, grid, stream))) return rc;
  }
  // ---- GEMM2: y = h . w2^T   (+ ys = hs . ws2^T)
  if (phases & 2) {
    CUtensorMap a0, b0, a1, b1;
    if ((rc = make_map_bf16(&a0, f->h, (uint64_t)f->capacity, (uint64_t)f->ip, gemm::BM))) return rc;
    if ((rc = make_map_bf16(&b0, f->w2, (uint64_t)f->num_experts_w * f->dp, (uint64_t)f->ip, gemm::BN))) return rc;
    if (shared) {
      if ((rc = make_map_bf16(&a1, f->hs, (uint64_t)f->shared_rows, (uint64_t)f->shared_ip, gemm::BM))) return rc;
      if ((rc = make_map_bf16(&b1, f->ws2, (uint64_t)f->dp, (uint64_t)f->shared_ip, gemm::BN))) return rc;
    } else {
      a1 = a0;
      b1 = b0;
    }
    gemm::Params p{};
    p.epi = gemm::kEpiStore;
    p.tile_counter = f->tile_counters != nullptr ? f->tile_counters + 2 : nullptr;  // GEMM2: [2, 4)
    p.err = f->err;
    p.nseg = shared ? 2 : 1;
    // the longer K first; with the fused return (ep_ctx) the routed tiles first, so that their
    // NVLink stores drain while the shared-expert tiles compute
    p.seg_first = (shared && f->shared_ip > f->ip && f->ep_ctx == nullptr) ? 1 : 0;
    p.l2_hints = f->cache_hints & 1;
    p.l2_ahead = (f->cache_hints >> 8) & 0xff;
    p.interleave_lead = (shared && routed && (f->tile_order & 1)) ? 0 : -1;
    gemm::set_weight_major(p, f->tile_order);
    p.ep_signal = routed ? static_cast<ep::Ctx*>(f->ep_ctx) : nullptr;
    gemm::Segment& s0 = p.seg[0];
    s0.ep = static_cast<const ep::Ctx*>(f->ep_ctx);
    s0.group_offsets = f->group_offsets;
    s0.group_weight = f->group_weight;
    s0.group_order = f->group_order;
    s0.ngroups = routed ? f->num_groups : 0;
    s0.rows = 0;
    s0.n_tiles = f->dp / gemm::BN;
    s0.b_rows_per_group = f->dp;
    s0.k_blocks = (f->ip + gemm::BK - 1) / gemm::BK;
    s0.c = reinterpret_cast<__nv_bfloat16*>(f->y);
    s0.ldc = f->d;
    s0.n_store = f->d;
    s0.capacity = f->capacity;
    if (shared) {
      gemm::Segment& s1 = p.seg[1];
      s1.group_offsets = nullptr;
      s1.group_weight = nullptr;
      s1.ngroups = 1;
      s1.rows = f->shared_rows;
      s1.n_tiles = f->dp / gemm::BN;
      s1.b_rows_per_group = f->dp;
      s1.k_blocks = (f->shared_ip + gemm::BK - 1) / gemm::BK;
      s1.c = reinterpret_cast<__nv_bfloat16*>(f->ys);
      s1.ldc = f->d;
      s1.n_store = f->d;
      s1.capacity = f->shared_rows;
    }
    if ((rc = launch_one(gemm::kEpiStore, a0, b0, a1, b1, p, grid, stream))) return rc;
  }
  return DSCA_OK;
}

// 2-D byte tensor map over a row-major [rows, cols] matrix (e4m3 weights or two-term token rows),
// box = box_rows x 128 bytes, 128-byte swizzle.
int make_map_e4m3(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  PFN_encodeTiled enc = get_encode_fn();
  if (enc == nullptr) return DSCA_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || cols % 16 != 0) return DSCA_ERR_BAD_ARG;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DSCA_OK : DSCA_ERR_CUDA;
}

// GEMM1 of the f8_split FFN on single-CTA tiles (128 tokens x 256 weight rows): h = act(a . w1^T),
// hs = act(xs . ws1^T) in bf16, the tokens as two-term e4m3 rows.
int launch_gemm1_f8_single(const dsca_ffn_args* f, int num_sms, cudaStream_t stream) {
  const int grid = f->num_ctas > 0 ? f->num_ctas : num_sms;
  const int segs = f->segments == 0 ? 3 : f->segments;
  const bool shared = f->shared_rows > 0 && (segs & 2);
  const bool routed = (segs & 1) != 0;
  if (!routed && !shared) return DSCA_OK;
  const int Kd = (f->d + 127) & ~127;
  int rc;
  CUtensorMap a0, b0, a1, b1;
  if ((rc = make_map_e4m3(&a0, f->a, (uint64_t)std::max(f->capacity, 1), (uint64_t)2 * Kd, gemm::BM))) return rc;
  if ((rc = make_map_e4m3(&b0, f->w1, (uint64_t)f->num_experts_w * f->n1p, (uint64_t)f->d, gemm::BN))) return rc;
  if (shared) {
    if ((rc = make_map_e4m3(&a1, f->xs, (uint64_t)f->shared_rows, (uint64_t)2 * Kd, gemm::BM))) return rc;
    if ((rc = make_map_e4m3(&b1, f->ws1, (uint64_t)f->shared_n1p, (uint64_t)f->d, gemm::BN))) return rc;
  } else {
    a1 = a0;
    b1 = b0;
  }
  gemm::Params p{};
  const int epi = f->act == DSCA_ACT_SWIGLU ? gemm::kEpiSwiGLU : gemm::kEpiReLU;
  p.epi = epi;
  p.tile_counter = f->tile_counters;  // GEMM1: [0, 2)
  p.err = f->err;
  p.nseg = shared ? 2 : 1;
  p.seg_first = 0;
  p.interleave_lead = -1;
  gemm::set_weight_major(p, f->tile_order);
  p.l2_hints = f->cache_hints & 1;
    p.l2_ahead = (f->cache_hints >> 8) & 0xff;
  gemm::Segment& s0 = p.seg[0];
  s0.group_offsets = f->group_offsets;
  s0.group_weight = f->group_weight;
  s0.group_order = f->group_order;
  s0.ngroups = routed ? f->num_groups : 0;
  s0.n_tiles = f->n1p / gemm::BN;
  s0.b_rows_per_group = f->n1p;
  s0.k_blocks = (f->d + 127) / 128;
  s0.c = reinterpret_cast<__nv_bfloat16*>(f->h);
  s0.ldc = f->ip;
  s0.n_store = f->ip;
  s0.capacity = f->capacity;
  s0.t_lo = Kd;
  s0.t_scale = f->a_scale;
  s0.w_scale = f->w1_scale;
  if (shared) {
    gemm::Segment& s1 = p.seg[1];
    s1.ngroups = 1;
    s1.rows = f->shared_rows;
    s1.n_tiles = f->shared_n1p / gemm::BN;
    s1.b_rows_per_group = f->shared_n1p;
    s1.k_blocks = (f->d + 127) / 128;
    s1.c = reinterpret_cast<__nv_bfloat16*>(f->hs);
    s1.ldc = f->shared_ip;
    s1.n_store = f->shared_ip;
    s1.capacity = f->shared_rows;
    s1.t_lo = Kd;
    s1.t_scale = f->xs_scale;
    s1.w_scale = f->ws1_scale;
  }
  return epi == gemm::kEpiSwiGLU ? launch_kernel<gemm::kEpiSwiGLU, true>(a0, b0, a1, b1, p, grid, stream)
                                 : launch_kernel<gemm::kEpiReLU, true>(a0, b0, a1, b1, p, grid, stream);
}

}  // namespace dsca
