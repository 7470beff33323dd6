// Wide-step FP8 block-sparse VSA attention (fine step) for sm_100a, included by vsa_attn.cu (it shares that file's
// arguments, helpers and status word).
//
// Same semantics as vsa_fp8_kernel with f16 V (E4M3 Q/K scores scaled by the per-tile Q/K scales, lazy-rescaled fp32
// online softmax, P in f16 scaled by sv_b / sv_head, O = (sum P' V') * sv_head / l, bf16 output, optional log2 LSE),
// with the key tiles of a query tile split into two streams by list parity (entries 0, 2, 4, ... and 1, 3, 5, ...),
// each with its own running maximum, sum and O accumulator, merged in the epilogue. A step takes four list entries:
// two key tiles of each stream (128 keys), scored and exponentiated together. Weight-stationary MMAs (tcgen05.mma.ws,
// M = 64) compute both streams at once on the whole 128-lane datapath:
//   S: .ws M=64 N=256 kind::f8f6f4, A = the query tile (64 x 128 E4M3), B = the step's four key tiles (stream 0's two,
//      then stream 1's two: 256 rows): stream 0's 128 scores per row land in TMEM lanes 0-63, stream 1's in lanes
//      64-127, 128 columns each.
//   PV: .ws M=64 N=256 kind::f16, A = P from TMEM (each lane half holds its stream's P, written over its S), B = one
//      f16 V tile of each stream side by side along N ([stream 0: d 0-63 | d 64-127 | stream 1: d 0-63 | d 64-127],
//      planes of 64 keys x 128 bytes): eight K=16 instructions per step (four per V tile), stream h accumulating into
//      its lanes' 128 columns of O.
// The tensor pipe executes a thread's MMAs in order and a commit covers everything issued before it, which the
// pipeline leans on: the S of step j+1 is issued after the PV of step j into the same TMEM columns (it overwrites P(j)
// only once PV(j) has read it), and when the softmax sees S(j) complete, PV(j-1) is complete too, so it may rescale O
// without a wait.
//
// Work item = (head, query tiles 2p and 2p+1), the two query tiles in flight together (tile m owns TMEM columns
// [256m, 256m+256): S/P at +0, O at +128) so one tile's softmax runs while the other's MMAs execute. A query tile with
// L selected key tiles takes max(1, ceil(L/4)) steps; a stream without a tile in a slot of a step computes on a
// duplicate of a listed tile with every key masked (P = 0). The lists are read from global memory by every role.
// CTA = 11 warps:
//   warp 0      TMA loads of Q (both tiles) and K (ring of 2 x 32 KB: the four key tiles of a step) in S order
//   warp 1      TMEM allocation; lane 0 issues the MMAs: S(0) of both tiles, then per step j and tile the PV of step
//               j (once its softmax wrote P) followed by the S of step j+1
//   warps 2-5   softmax of query tile 0, warps 6-9 of tile 1: one thread per TMEM lane, i.e. per (stream, row); the
//               epilogue merges the two streams of each row through shared memory and stores the bf16 rows
//   warp 10     TMA loads of f16 V (ring of 4 x 32 KB: one key tile of each stream) in PV order
// Every wait is bounded (kLimitNs) and records H3B_ETIMEOUT in the attention status word.

namespace ws {
constexpr int KST = 2;   // K ring slots: the four E4M3 key tiles of a step (256 rows x 128 B)
constexpr int VST = 4;   // V ring slots: one f16 key tile of each stream as four planes of 64 keys x 128 B
constexpr int WARPS = 11;
constexpr int THREADS = WARPS * 32;
constexpr int K_SLOT = 4 * TILE * D;
constexpr int V_PLANE = TILE * 128;
constexpr int V_SLOT = 4 * V_PLANE;
// score of a masked key (past a tile's length, or a slot with no tile): finite, below any E4M3 dot product (|S| <=
// 128 * 448 * 448 < 2.6e7) by far, and still finite once multiplied by a Q/K scale coefficient (< 1e8)
constexpr float kMaskedScore = -1.0e30f;

struct __align__(1024) Smem {
  uint8_t q[2][TILE * D];            // [query tile] E4M3, 128-byte swizzle
  uint8_t k[KST][K_SLOT];            // [slot] key tiles: stream 0's first and second, stream 1's first and second
  uint8_t v[VST][V_SLOT];            // [slot] planes (stream, half of d): 64 keys x 64 f16, 128-byte swizzle
  float4 xo[2][2][64][4];            // [query tile][receiving stream][row][16-byte chunk] epilogue exchange
  uint64_t q_full, q_empty;
  uint64_t k_full[KST], k_empty[KST], v_full[VST], v_empty[VST];
  uint64_t s_full[2], p_full[2];     // [query tile]
  uint64_t o_last[2], o_free[2];     // [query tile] the item's last PV completed / the epilogue has read O
  uint64_t xchg[2];                  // [query tile] the epilogue's exchange points (the tile's four warps)
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ void mma_ws_e4m3(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.ws.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_ws_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                              uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.ws.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_16cols(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// A query tile's list as every role reads it: its length (clamped to the list stride, and to L_MAX), and the key tile
// of stream hs in slot t of step j (entry 4j + 2t + hs; a duplicate of the first entry, masked by the softmax, where
// the list has none)
struct TileList {
  const int32_t* row;
  int n;
  __device__ TileList(const AttnArgs& a, int h, int t) {
    row = a.idx + ((size_t)h * a.n_q_ext + t) * a.idx_ld;
    n = min(min(max(a.num[(size_t)h * a.n_q_ext + t], 0), a.idx_ld), L_MAX);
  }
  __device__ int steps() const { return max(1, (n + 3) >> 2); }
  __device__ bool has(int j, int hs, int t) const { return 4 * j + 2 * t + hs < n; }
  __device__ int tile(const AttnArgs& a, int j, int hs, int t) const {
    const int e = 4 * j + 2 * t + hs;
    const int v = e < n ? row[e] : (n > 0 ? row[0] : 0);
    return min(max(v, 0), a.n_kv - 1);
  }
};
}  // namespace ws

__global__ void __launch_bounds__(ws::THREADS, 1)
    vsa_ws_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  using namespace ws;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  ws::Smem& sm = *reinterpret_cast<ws::Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort_flag = &sm.abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_empty, 1);  // the item's last S MMA
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.p_full[i], 4);  // the tile's four softmax warps
      mbar_init(&sm.o_last[i], 1);
      mbar_init(&sm.o_free[i], 4);
      mbar_init(&sm.xchg[i], 4);
    }
    for (int s = 0; s < KST; ++s) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_empty[s], 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.v_empty[s], 1);
    }
    mbar_init(&sm.drain, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const int pairs = a.n_q_ext / 2;

  if (warp == 0) {
    // -------------------------------------------------------------- Q and K producer (lane 0)
    if (lane == 0) {
      uint32_t q_phase = 0, kc = 0;  // kc: K ring uses so far
      bool ok = true;
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x) {
        const int h = item / pairs, p = item - h * pairs;
        const TileList L[2] = {TileList(a, h, 2 * p), TileList(a, h, 2 * p + 1)};
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          const int want = a.num[(size_t)h * a.n_q_ext + 2 * p + s];
          if (min(want, a.idx_ld) > L_MAX) atomicExch(&g_attn_status, H3B_EINVAL);
        }
        auto load_k = [&](int s, int j) -> bool {
          const int slot = (int)(kc % KST);
          if (!mbar_wait_bounded(&sm.k_empty[slot], ((kc / KST) & 1u) ^ 1u, abort_flag, kLimitNs)) return false;
          mbar_arrive_expect_tx(&sm.k_full[slot], K_SLOT);
#pragma unroll
          for (int hs = 0; hs < 2; ++hs)
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const int b = L[s].tile(a, j, hs, t);
              tma_load_3d(&sm.k[slot][(2 * hs + t) * TILE * D], &tmK, 0, (b % a.tpc_kv) * TILE,
                          (b / a.tpc_kv) * a.heads + h, &sm.k_full[slot]);
            }
          ++kc;
          return true;
        };
        if (!mbar_wait_bounded(&sm.q_empty, q_phase ^ 1u, abort_flag, kLimitNs)) {
          ok = false;
        } else {
          q_phase ^= 1u;
          mbar_arrive_expect_tx(&sm.q_full, 2 * TILE * D);
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            const int t = 2 * p + s;
            tma_load_3d(&sm.q[s][0], &tmQ, 0, (t % a.tpc_q) * TILE, (t / a.tpc_q) * a.heads + h, &sm.q_full);
          }
          // the order the MMA thread consumes them: S(0) of both tiles, then per step j and tile s the S of step j+1
          const int st[2] = {L[0].steps(), L[1].steps()};
          ok = load_k(0, 0) && load_k(1, 0);
          const int steps = max(st[0], st[1]);
          for (int j = 0; j < steps && ok; ++j) {
#pragma unroll
            for (int s = 0; s < 2; ++s) {
              if (!ok || j + 1 >= st[s]) continue;
              ok = load_k(s, j + 1);
            }
          }
        }
        if (!ok) fail_cta(abort_flag);
      }
      if (!ok) {
        // aborted: let the copies already issued land before the CTA exits (the ring's last uses, short bounds)
        volatile int no_abort = 0;
        for (uint32_t u = kc > (uint32_t)KST ? kc - KST : 0u; u < kc; ++u)
          mbar_wait_bounded(&sm.k_full[u % KST], (u / KST) & 1u, &no_abort, kLimitNs / 64);
      }
    }
  } else if (warp == WARPS - 1) {
    // -------------------------------------------------------------- V producer (lane 0): f16 V tiles in PV order
    if (lane == 0) {
      uint32_t vc = 0;  // V ring uses so far
      bool ok = true;
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x) {
        const int h = item / pairs, p = item - h * pairs;
        const TileList L[2] = {TileList(a, h, 2 * p), TileList(a, h, 2 * p + 1)};
        auto load_v = [&](int s, int j, int t) -> bool {
          const int slot = (int)(vc % VST);
          if (!mbar_wait_bounded(&sm.v_empty[slot], ((vc / VST) & 1u) ^ 1u, abort_flag, kLimitNs)) return false;
          mbar_arrive_expect_tx(&sm.v_full[slot], V_SLOT);
#pragma unroll
          for (int hs = 0; hs < 2; ++hs) {
            const int b = L[s].tile(a, j, hs, t);
#pragma unroll
            for (int dh = 0; dh < 2; ++dh)
              tma_load_3d(&sm.v[slot][(2 * hs + dh) * V_PLANE], &tmV, 128 * dh, (b % a.tpc_kv) * TILE,
                          (b / a.tpc_kv) * a.heads + h, &sm.v_full[slot]);
          }
          ++vc;
          return true;
        };
        const int st[2] = {L[0].steps(), L[1].steps()};
        const int steps = max(st[0], st[1]);
        for (int j = 0; j < steps && ok; ++j) {
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            if (!ok || j >= st[s]) continue;
            ok = load_v(s, j, 0) && load_v(s, j, 1);
          }
        }
        if (!ok) fail_cta(abort_flag);
      }
      if (!ok) {
        volatile int no_abort = 0;
        for (uint32_t u = vc > (uint32_t)VST ? vc - VST : 0u; u < vc; ++u)
          mbar_wait_bounded(&sm.v_full[u % VST], (u / VST) & 1u, &no_abort, kLimitNs / 64);
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = idesc_mn(TILE, 4 * TILE, false);  // M = 64 (.ws), N = 256: the step's four key tiles
      const uint32_t idesc_pv = idesc_mn(TILE, 2 * D, true);     // M = 64 (.ws), N = 256: both streams' O
      uint32_t q_phase = 0, kc = 0, vc = 0;
      uint32_t pfc[2] = {0u, 0u}, ofc[2] = {0u, 0u};  // per tile: P signals taken, O-free signals taken
      bool ok = true;
      int it = 0;
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++it) {
        const int h = item / pairs, p = item - h * pairs;
        const int st[2] = {TileList(a, h, 2 * p).steps(), TileList(a, h, 2 * p + 1).steps()};
        const int total_s = st[0] + st[1];
        int issued_s = 0;
        if (!mbar_wait_bounded(&sm.q_full, q_phase, abort_flag, kLimitNs)) {
          fail_cta(abort_flag);
          break;
        }
        q_phase ^= 1u;
        tc_fence_after();
        const uint64_t dq[2] = {desc_k_sw128(smem_addr(&sm.q[0][0])), desc_k_sw128(smem_addr(&sm.q[1][0]))};
        auto issue_s = [&](int s) -> bool {
          const int slot = (int)(kc % KST);
          if (!mbar_wait_bounded(&sm.k_full[slot], (kc / KST) & 1u, abort_flag, kLimitNs)) return false;
          tc_fence_after();
          const uint64_t dk = desc_k_sw128(smem_addr(&sm.k[slot][0]));
#pragma unroll
          for (int i = 0; i < 4; ++i) ws::mma_ws_e4m3(tmem + 256u * s, dq[s] + 2 * i, dk + 2 * i, idesc_s, i != 0);
          tc_commit(&sm.k_empty[slot]);
          tc_commit(&sm.s_full[s]);
          ++kc;
          if (++issued_s == total_s) tc_commit(&sm.q_empty);
          return true;
        };
        auto issue_pv = [&](int s, int j) -> bool {
          if (!mbar_wait_bounded(&sm.p_full[s], pfc[s] & 1u, abort_flag, kLimitNs)) return false;
          ++pfc[s];
          if (j == 0 && it > 0) {  // the previous item's epilogue has read this tile's O
            if (!mbar_wait_bounded(&sm.o_free[s], ofc[s] & 1u, abort_flag, kLimitNs)) return false;
            ++ofc[s];
          }
#pragma unroll
          for (int t = 0; t < 2; ++t) {  // one V tile of each stream: K = 16 keys per MMA (8 TMEM columns of P)
            const int slot = (int)(vc % VST);
            if (!mbar_wait_bounded(&sm.v_full[slot], (vc / VST) & 1u, abort_flag, kLimitNs)) return false;
            tc_fence_after();
            const uint64_t dv = desc_mn_sw128(smem_addr(&sm.v[slot][0]), V_PLANE);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              ws::mma_ws_f16_ts(tmem + 256u * s + 128u, tmem + 256u * s + 8u * (4 * t + i),
                                dv + (uint64_t)((i * 16 * 128) >> 4), idesc_pv, (j > 0 || t > 0 || i > 0) ? 1u : 0u);
            tc_commit(&sm.v_empty[slot]);
            ++vc;
          }
          return true;
        };
        ok = issue_s(0) && issue_s(1);
        const int steps = max(st[0], st[1]);
        for (int j = 0; j < steps && ok; ++j) {
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            if (!ok || j >= st[s]) continue;
            ok = issue_pv(s, j);
            if (ok && j + 1 == st[s]) tc_commit(&sm.o_last[s]);
            if (ok && j + 1 < st[s]) ok = issue_s(s);
          }
        }
        if (!ok) {
          fail_cta(abort_flag);
          break;
        }
      }
      tc_commit(&sm.drain);
      volatile int no_abort = 0;
      if (!mbar_wait_bounded(&sm.drain, 0, &no_abort, kLimitNs)) fail_cta(abort_flag);
    }
  } else {
    // -------------------------------------------------------------- softmax of one query tile + epilogue
    const int m = (warp - 2) >> 2;         // query tile of the pair
    const int q4 = warp & 3;               // TMEM lane quarter this warp may access
    const int hs = q4 >> 1;                // stream (lane half)
    const int r = 32 * (q4 & 1) + lane;    // row of the query tile
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t cS = 256u * m, cO = 256u * m + 128u;
    uint32_t sph = 0, olc = 0, xph = 0;
    // an exchange point of the tile's four warps (an mbarrier with a bounded wait, not a named barrier: a warp that
    // gave up must not leave the others waiting for good)
    auto group_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.xchg[m]);
      const bool got = warp_wait_bounded(&sm.xchg[m], xph & 1u, abort_flag, lane);
      ++xph;
      return got;
    };
    bool ok = true;
    for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x) {
      const int h = item / pairs, p = item - h * pairs;
      const int tq = 2 * p + m;
      const TileList L(a, h, tq);
      const int steps = L.steps();
      const float qcoef = a.coef * (a.qs ? a.qs[(size_t)h * a.q_scale_ld + tq] : 1.f);
      const float* ksh = a.ks ? a.ks + (size_t)h * a.kv_scale_ld : nullptr;
      const float* vsh = a.vs + (size_t)h * a.kv_scale_ld;
      const float inv_vhead = 1.f / a.vs_head[h];
      float m_ref = -INFINITY, l = 0.f;
      // per-tile scalars of this stream's two key tiles of a step, loaded one step ahead
      int vbs_n[2];
      float ks_n[2], vs_n[2];
      auto fetch = [&](int j) {
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          vbs_n[t] = 0;  // every key masked where the stream has no tile in this slot
          ks_n[t] = 1.f;
          vs_n[t] = 0.f;
          if (j < steps && L.has(j, hs, t)) {
            const int b = L.tile(a, j, hs, t);
            vbs_n[t] = a.vbs_kv[b];
            vs_n[t] = vsh[b];
            if (ksh) ks_n[t] = ksh[b];
          }
        }
      };
      fetch(0);
      for (int j = 0; j < steps; ++j) {
        const int vbs_j0 = vbs_n[0], vbs_j1 = vbs_n[1];
        const float ks_j0 = ks_n[0], ks_j1 = ks_n[1], vs_j0 = vs_n[0], vs_j1 = vs_n[1];
        fetch(j + 1);
        if (!warp_wait_bounded(&sm.s_full[m], sph & 1u, abort_flag, lane)) {
          ok = false;
          break;
        }
        ++sph;
        tc_fence_after();
        // two passes over the step's 128 scores (64 at a time, to stay within the registers of 11 warps): the row
        // maximum, then the exponentials from a second read of the same columns
        // (the per-tile scalars are picked with selects: a runtime index into the small arrays would put them in
        // local memory, which the 64-column mask below would then reload per column)
        // Keys past a tile's length are left out per 8-column chunk: chunk k counts if 8k < vbt (a warp-uniform
        // predicate, since every lane of a warp has the same key tile), in the row maximum as a selected chunk
        // maximum and in P as a mask word ANDed into the chunk's four packed pairs before they are summed. A length
        // that is not a multiple of 8 first sets the scores of its partial chunk's tail to a sentinel (a per-element
        // select, on those tiles only).
        auto load_tile = [&](int t, uint32_t (&st)[64]) {
          tmem_ld_32cols(tmem + lane_off + cS + 64u * t, *reinterpret_cast<uint32_t(*)[32]>(&st[0]));
          tmem_ld_32cols(tmem + lane_off + cS + 64u * t + 32u, *reinterpret_cast<uint32_t(*)[32]>(&st[32]));
          tmem_ld_wait();
          const int vbt = t ? vbs_j1 : vbs_j0;
          if (vbt & 7) {
            const uint32_t masked = __float_as_uint(kMaskedScore);
#pragma unroll
            for (int c = 0; c < 64; ++c) st[c] = c >= vbt ? masked : st[c];
          }
        };
        float mx = -INFINITY;
#pragma unroll 1
        for (int t = 0; t < 2; ++t) {
          uint32_t st[64];
          load_tile(t, st);
          const int vbt = t ? vbs_j1 : vbs_j0;
          float mraw = kMaskedScore;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t* c8 = st + 8 * k;
            const float cm = fmaxf(fmax3(__uint_as_float(c8[0]), __uint_as_float(c8[1]), __uint_as_float(c8[2])),
                                   fmax3(__uint_as_float(c8[3]), __uint_as_float(c8[4]),
                                         fmaxf(__uint_as_float(c8[5]), fmaxf(__uint_as_float(c8[6]),
                                                                             __uint_as_float(c8[7])))));
            mraw = 8 * k < vbt ? fmaxf(mraw, cm) : mraw;
          }
          if (mraw > kMaskedScore) mx = fmaxf(mx, mraw * (qcoef * (t ? ks_j1 : ks_j0)));  // coef > 0
        }
        const bool grow = mx > m_ref + RESCALE_LOG2;
        const bool had_mass = m_ref != -INFINITY;
        float alpha = 1.f;
        if (grow) {
          alpha = had_mass ? ex2(m_ref - mx) : 1.f;
          m_ref = mx;
        }
        // PV(j-1) completed before S(j) did (issued before it, in order), so O is quiet until this step's signal
        if (__any_sync(0xffffffffu, grow && had_mass)) {
#pragma unroll 1
          for (int c0 = 0; c0 < D; c0 += 32) {
            uint32_t o[32];
            tmem_ld_32cols(tmem + lane_off + cO + c0, o);
            tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
            tmem_st_32cols(tmem + lane_off + cO + c0, o);
          }
        }
        l *= alpha;
#pragma unroll 1
        for (int t = 0; t < 2; ++t) {
          uint32_t pw[32];
          if (m_ref == -INFINITY) {
#pragma unroll
            for (int c = 0; c < 32; ++c) pw[c] = 0u;
          } else {
            uint32_t st[64];
            load_tile(t, st);
            const float coef = qcoef * (t ? ks_j1 : ks_j0);
            uint32_t acc[4] = {0u, 0u, 0u, 0u};
            const __half2 vr2 = __float2half2_rn((t ? vs_j1 : vs_j0) * inv_vhead);  // P' = P * sv_b / sv_head
            const uint32_t vr = *reinterpret_cast<const uint32_t*>(&vr2);
            const uint64_t coef2 = pack_f32x2(coef, coef), nb2 = pack_f32x2(-m_ref, -m_ref);
            const int vbt = t ? vbs_j1 : vbs_j0;
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const uint32_t keep = 8 * (c >> 2) < vbt ? 0xFFFFFFFFu : 0u;  // chunk c/4 of the tile's 8 chunks
              const uint32_t e = ex2_pair(st[2 * c], st[2 * c + 1], coef2, nb2) & keep;
              acc[c & 3] = hadd2(acc[c & 3], e);
              pw[c] = hmul2(e, vr);
            }
            const float2 s0 = __half22float2(*reinterpret_cast<const __half2*>(&acc[0]));
            const float2 s1 = __half22float2(*reinterpret_cast<const __half2*>(&acc[1]));
            const float2 s2 = __half22float2(*reinterpret_cast<const __half2*>(&acc[2]));
            const float2 s3 = __half22float2(*reinterpret_cast<const __half2*>(&acc[3]));
            l += ((s0.x + s0.y) + (s1.x + s1.y)) + ((s2.x + s2.y) + (s3.x + s3.y));
          }
          tmem_st_32cols(tmem + lane_off + cS + 32u * t, pw);  // P over this step's S columns
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_full[m]);
      }
      if (!ok) break;
      // ---- epilogue: the item's last PV, then merge the two streams of each row
      if (!warp_wait_bounded(&sm.o_last[m], olc & 1u, abort_flag, lane)) break;
      ++olc;
      tc_fence_after();
      sm.xo[m][hs ^ 1][r][0] = make_float4(m_ref, l, 0.f, 0.f);
      if (!group_sync()) break;
      const float4 ml = sm.xo[m][hs][r][0];
      if (!group_sync()) break;  // read before the first pass overwrites it
      const float m_other = ml.x, l_other = ml.y;
      const float m0 = hs ? m_other : m_ref, m1 = hs ? m_ref : m_other;
      const float l0 = hs ? l_other : l, l1 = hs ? l : l_other;
      const float M = fmaxf(m0, m1);
      const float f0 = (M == -INFINITY || m0 == -INFINITY) ? 0.f : ex2(m0 - M);
      const float f1 = (M == -INFINITY || m1 == -INFINITY) ? 0.f : ex2(m1 - M);
      const float Lsum = l0 * f0 + l1 * f1;
      const float oscale = Lsum > 0.f ? a.vs_head[h] / Lsum : 0.f;
      const float g = (hs ? f1 : f0) * oscale;  // this stream's weight in the row
      const bool row_ok = r < a.vbs_q[tq];
      const size_t orow =
          (size_t)((tq / a.tpc_q) * a.heads + h) * (size_t)a.rows_chunk_q + (size_t)(tq % a.tpc_q) * TILE + r;
      // stream hs writes output columns 64*hs .. 64*hs+63: per 16-column pass it sends its weighted O of the other
      // stream's columns through shared memory (16-byte chunks rotated by row) and adds the other stream's part of
      // its own columns
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t send[16], own[16];
        ws::tmem_ld_16cols(tmem + lane_off + cO + 64u * (hs ^ 1) + 16u * c, send);
        ws::tmem_ld_16cols(tmem + lane_off + cO + 64u * hs + 16u * c, own);
        tmem_ld_wait();
        if (c == 3) {  // O read: the next item's PV MMAs of this tile may overwrite it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.o_free[m]);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k)  // a stream with no mass contributes nothing
          sm.xo[m][hs ^ 1][r][k ^ (r & 3)] =
              g != 0.f ? make_float4(__uint_as_float(send[4 * k]) * g, __uint_as_float(send[4 * k + 1]) * g,
                                     __uint_as_float(send[4 * k + 2]) * g, __uint_as_float(send[4 * k + 3]) * g)
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        if (!group_sync()) {
          ok = false;
          break;
        }
        uint32_t pk[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float4 u = sm.xo[m][hs][r][k ^ (r & 3)];
          const float add[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int cc = 4 * k + 2 * e;
            const float x0 = (g != 0.f ? __uint_as_float(own[cc]) * g : 0.f) + add[2 * e];
            const float x1 = (g != 0.f ? __uint_as_float(own[cc + 1]) * g : 0.f) + add[2 * e + 1];
            pk[2 * k + e] = row_ok ? pack_bf16x2(x0, x1) : 0u;
          }
        }
        uint4* dst = reinterpret_cast<uint4*>(a.out + orow * D + 64 * hs + 16 * c);
        dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        if (!group_sync()) {  // the buffer is read before the next pass (or the next item) writes it
          ok = false;
          break;
        }
      }
      if (!ok) break;
      if (a.lse && row_ok && hs == 0) a.lse[orow] = Lsum > 0.f ? M + __log2f(Lsum) : -INFINITY;
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
