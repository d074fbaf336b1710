// Shared by the tcgen05 GEMM kernels (gemm_tcgen05.cu: tile-per-CTA kernel with
// split-K and the swapped decode mode; gemm_persistent.cu: persistent kernel
// for prefill-sized problems): argument block, tile constants and the
// normal-mode (activations = A operand) epilogue.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace braid {

// Fused QKV epilogue (epi == 2): per-head q/k RMSNorm, RoPE on k, q written
// unrotated to q_out, k/v appended to the paged KV cache at slots[token].
struct QkvEpi {
  __nv_bfloat16* q_out;  // [T, Hq, D]
  __nv_bfloat16* kv;     // layer cache [P, 2, Hkv, PS, D]
  const int* slots;
  const int* positions;
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  const float* cos;
  const float* sin;
  int Hq, Hkv, D, PS, use_rope;
  float eps;
  int num_slots;  // pages * PS of the cache (checked build)
  int rope_len;   // rows of cos/sin (checked build)
};

// Push epilogue (epi == 3, swapped mode): the bf16 result tile is written to
// every tensor-parallel peer's receive area (slot epoch & 1, source row rank)
// instead of local memory, then each peer's arrival counter for this rank is
// bumped; tp_reduce_add in comm.cu completes the all-reduce.
//
// Fused all-reduce (fused == 1): the same push, then per 128-feature tile a
// release flag (value epoch + 1) in every peer's tile_flags[rank][tile]; the
// tile's CTA waits (bounded) until every source's flag for this tile reached
// epoch + 1, sums the tp received tiles in fp32, adds the residual and writes
// the result in place.  The last tile to finish advances the epoch
// (epoch_state[2] counts finished tiles).  All CTAs of the grid are resident
// at once (the split factor keeps the grid within one wave), so the per-tile
// waits cannot block a CTA that has not started.
struct PushEpi {
  const uint64_t* peers;       // [tp] base addresses of the peers' comm buffers
  int64_t flags_off;           // byte offset of the arrival counters in a comm buffer
  uint64_t* epoch_state;       // local [0] epoch (completed all-reduce calls), [2] finished tiles
  int rank, tp, maxT;
  int fused;                   // 1: wait for the peers' tiles and reduce in this kernel
  int64_t tile_flags_off;      // byte offset of u64 tile_flags[tp][max_tiles]
  int max_tiles;
  int* status;                 // comm status word {code, rank, peer, epoch}
  uint64_t timeout_ns;
};

// Sequence-parallel tensor parallelism for prefill-sized batches.  Token rows
// are owned by ranks in contiguous blocks of rows_per_rank.  Comm-buffer
// regions (byte offsets, identical on every rank):
//   recv_off      bf16 [tp source][rows_per_rank][H]: partial rows pushed to their owner
//   rs_flags_off  u64 [tp]: per-source count of partial tiles received (cumulative)
//   ag_flags_off  u64 [tp]: per-owner count of gathered-row blocks received (cumulative)
// Reduce-scatter epilogue (epi == 4, normal mode): each output row is stored
// into its owner's recv slot for this source, then the owner's rs counter for
// this rank is bumped once per tile.  All-gather wait: before the A tile of
// rows [m0, m0+128) is loaded, the ag counter of every owner of those rows
// must reach ag_expected (0 = no wait); the owners' reduce kernel
// (sp_reduce_allgather in comm.cu) pushed those rows and their 1/rms.
struct SpArgs {
  const uint64_t* peers;  // [tp] comm buffer bases (device array)
  int64_t recv_off, rs_flags_off, ag_flags_off;
  uint64_t ag_expected;
  int* status;            // comm status word {code, rank, peer, n}
  uint64_t timeout_ns;
  int rank, tp, rows_per_rank, H;
};

struct GemmArgs {
  int M, N, K;        // A rows, B rows, reduction length
  int swap;           // 1: A is the weight, output written transposed
  int epi;            // 0 plain, 1 swiglu, 2 qkv, 3 push (all-reduce), 4 push to row owner (reduce-scatter)
  __nv_bfloat16* out;
  int ldo;
  const __nv_bfloat16* bias;      // indexed by feature
  const __nv_bfloat16* residual;  // same layout as out
  int ldr;
  // Fused input RMSNorm: the norm weight is folded into the weight matrix and
  // each token's 1/rms(x) is applied here (x = the activation operand), either
  // computed in the epilogue from rs_x or read from rs_vec (precomputed).
  const __nv_bfloat16* rs_x;
  int rs_ld;
  float rs_eps;
  const float* rs_vec;
  int splits;
  int kb_per_split;
  int cluster;        // 1: the split-K CTAs of a tile form one cluster and reduce through DSMEM
  float* ws;          // split-K partials (global path)
  int* counters;      // one per output tile, kept at zero between launches
  int* err;           // error flag (bounded-wait timeout)
  QkvEpi qkv;
  PushEpi push;
  SpArgs sp;
  unsigned long long* trace;  // optional per-CTA phase timestamps (profiling)
  unsigned long long* span;   // optional launch span (profiling)
  PrefetchArgs pf;            // next GEMM's weight to pull into L2 (third tensor map)
};

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int XCH_LD = 17;  // exchange tile: 128 rows x 16 columns (+1 pad) fp32

// Wait (bounded) until every owner of rows [row0, row1) has pushed them.
// Generic-proxy stores from peers must be ordered before this thread's later
// TMA (async-proxy) reads, hence the proxy fence after the acquire loads.
BRAID_DEVICE bool sp_wait_rows(const SpArgs& sp, int row0, int row1) {
  if (sp.ag_expected == 0 || row1 <= row0) return true;
  const uint64_t* flags =
      reinterpret_cast<const uint64_t*>(reinterpret_cast<const char*>(sp.peers[sp.rank]) + sp.ag_flags_off);
  const int o0 = row0 / sp.rows_per_rank, o1 = (row1 - 1) / sp.rows_per_rank;
  for (int o = o0; o <= o1; ++o) {
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys_u64(flags + o) < sp.ag_expected) {
      if (globaltimer_ns() - t0 > sp.timeout_ns) {
        if (atomicCAS(sp.status, 0, 2) == 0) {
          sp.status[1] = sp.rank;
          sp.status[2] = o;
          sp.status[3] = (int)sp.ag_expected;
        }
        return false;
      }
      __nanosleep(32);
    }
  }
  fence_proxy_async_global();
  return true;
}

// Normal-mode epilogue of one 128 x BN tile: this thread owns tile row r
// (token m0 + r).  load_cols(c0, v) yields columns [c0, c0+16) of the row in
// fp32 with 1/rms and bias applied.  Called by the 128 epilogue threads together.
template <int BN, typename LoadCols>
BRAID_DEVICE void store_tile_normal(const GemmArgs& args, int m0, int n0, int r, LoadCols&& load_cols) {
  const int m = m0 + r;
  if (args.epi == 0) {
    for (int c0 = 0; c0 < BN; c0 += 16) {
      float v[16];
      load_cols(c0, v);
      if (m >= args.M) continue;
      __nv_bfloat16* o = args.out + (size_t)m * args.ldo + n0 + c0;
      const __nv_bfloat16* res = args.residual ? args.residual + (size_t)m * args.ldr + n0 + c0 : nullptr;
      const bool vec = n0 + c0 + 16 <= args.N &&
                       ((reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(res)) & 15) == 0;
      if (vec) {
        // 16 outputs = two 16-byte stores (the row is this thread's)
        uint4 rv[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
        if (res) {
          rv[0] = *reinterpret_cast<const uint4*>(res);
          rv[1] = *reinterpret_cast<const uint4*>(res + 8);
        }
        const __nv_bfloat16* re = reinterpret_cast<const __nv_bfloat16*>(rv);
        uint4 ov[2];
        __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(ov);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float y = rbf(v[j]);
          if (res) y += bf2f(re[j]);
          oe[j] = f2bf(y);
        }
        *reinterpret_cast<uint4*>(o) = ov[0];
        *reinterpret_cast<uint4*>(o + 8) = ov[1];
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (n0 + c0 + j < args.N) {
            float y = rbf(v[j]);
            if (res) y += bf2f(res[j]);
            o[j] = f2bf(y);
          }
        }
      }
    }
  } else if (args.epi == 4) {
    // Reduce-scatter push: row m -> recv[rank][m - owner*rows_per_rank] of its owner.
    const SpArgs& sp = args.sp;
    __nv_bfloat16* dst = nullptr;
    if (m < args.M) {
      const int own = m / sp.rows_per_rank;
      dst = reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<char*>(sp.peers[own]) + sp.recv_off) +
            ((size_t)sp.rank * sp.rows_per_rank + (m - own * sp.rows_per_rank)) * sp.H + n0;
    }
    for (int c0 = 0; c0 < BN; c0 += 16) {
      float v[16];
      load_cols(c0, v);
      if (dst == nullptr) continue;
      uint4 ov[2];
      __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(ov);
#pragma unroll
      for (int j = 0; j < 16; ++j) oe[j] = f2bf(v[j]);
      if (n0 + c0 + 16 <= args.N) {
        *reinterpret_cast<uint4*>(dst + c0) = ov[0];
        *reinterpret_cast<uint4*>(dst + c0 + 8) = ov[1];
      } else {
        for (int j = 0; j < 16; ++j)
          if (n0 + c0 + j < args.N) dst[c0 + j] = oe[j];
      }
    }
    __threadfence_system();
    named_bar_sync(1, 128);
    if (r == 0) {
      __threadfence_system();
      const int o0 = m0 / sp.rows_per_rank, o1 = (min(m0 + BM, args.M) - 1) / sp.rows_per_rank;
      for (int o = o0; o <= o1; ++o)
        atomicAdd(reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(sp.peers[o]) + sp.rs_flags_off) +
                      sp.rank, 1ull);
    }
  } else if (args.epi == 1) {
    // SwiGLU: per 128-column block, gate = cols [0,64), up = [64,128).
    for (int blk = 0; blk < BN / 128; ++blk) {
      for (int c0 = 0; c0 < 64; c0 += 16) {
        float g[16], u[16];
        load_cols(blk * 128 + c0, g);
        load_cols(blk * 128 + 64 + c0, u);
        if (m >= args.M) continue;
        const int f0 = (n0 + blk * 128) / 2 + c0;
        __nv_bfloat16* o = args.out + (size_t)m * args.ldo + f0;
        uint4 ov[2];
        __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(ov);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float gg = rbf(g[j]), uu = rbf(u[j]);
          const float sg = rbf(gg / (1.f + __expf(-gg)));
          oe[j] = f2bf(sg * uu);
        }
        if (2 * (f0 + 16) <= args.N && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
          *reinterpret_cast<uint4*>(o) = ov[0];
          *reinterpret_cast<uint4*>(o + 8) = ov[1];
        } else {
          for (int j = 0; j < 16; ++j)
            if (2 * (f0 + j) < args.N) o[j] = oe[j];
        }
      }
    }
  } else {
    // QKV: this thread owns token row m and whole heads of the tile.
    const QkvEpi& q = args.qkv;
    const int D = q.D;
    for (int hl = 0; hl < BN / D; ++hl) {
      const int col0 = hl * D;
      if (n0 + col0 >= args.N) break;
      const int head = (n0 + col0) / D;
      const bool is_q = head < q.Hq, is_k = !is_q && head < q.Hq + q.Hkv;
      const __nv_bfloat16* nw = is_q ? q.q_norm : (is_k ? q.k_norm : nullptr);
      float hr = 1.f;
      if (nw != nullptr) {
        float ss = 0.f;
        for (int c = 0; c < D; c += 16) {
          float v[16];
          load_cols(col0 + c, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float y = rbf(v[j]);
            ss += y * y;
          }
        }
        hr = rsqrtf(ss / D + q.eps);
      }
      // rows past M still take part in every load_cols (TMEM loads are warp-wide)
      __nv_bfloat16* dst = nullptr;
      int pos = 0;
      if (m < args.M) {
        if (is_q) {
          dst = q.q_out + ((size_t)m * q.Hq + head) * D;
        } else {
          const int slot = q.slots[m];
          const int kh = is_k ? head - q.Hq : head - q.Hq - q.Hkv;
          if (BRAID_IN_BOUNDS(slot >= 0 && slot < q.num_slots, 1, slot))
            dst = q.kv + ((((size_t)(slot / q.PS)) * 2 + (is_k ? 0 : 1)) * q.Hkv + kh) * q.PS * (size_t)D +
                  (size_t)(slot % q.PS) * D;
        }
        pos = q.positions[m];
        if (is_k && q.use_rope && !BRAID_IN_BOUNDS(pos >= 0 && pos < q.rope_len, 2, pos)) pos = 0;
      }
      for (int c = 0; c < D / 2; c += 16) {
        float a[16], b[16];
        load_cols(col0 + c, a);
        load_cols(col0 + D / 2 + c, b);
        if (dst == nullptr) continue;
        uint4 w1[2], w2[2];
        __nv_bfloat16* e1 = reinterpret_cast<__nv_bfloat16*>(w1);
        __nv_bfloat16* e2 = reinterpret_cast<__nv_bfloat16*>(w2);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float x1 = rbf(a[j]), x2 = rbf(b[j]);
          if (nw != nullptr) {
            x1 = rbf(rbf(x1 * hr) * bf2f(nw[c + j]));
            x2 = rbf(rbf(x2 * hr) * bf2f(nw[D / 2 + c + j]));
          }
          if (is_k && q.use_rope) {
            const float cs = q.cos[(size_t)pos * (D / 2) + c + j], sn = q.sin[(size_t)pos * (D / 2) + c + j];
            const float y1 = x1 * cs - x2 * sn, y2 = x2 * cs + x1 * sn;
            x1 = y1;
            x2 = y2;
          }
          e1[j] = f2bf(x1);
          e2[j] = f2bf(x2);
        }
        // head rows are 16-byte aligned (D and c are multiples of 8)
        *reinterpret_cast<uint4*>(dst + c) = w1[0];
        *reinterpret_cast<uint4*>(dst + c + 8) = w1[1];
        *reinterpret_cast<uint4*>(dst + D / 2 + c) = w2[0];
        *reinterpret_cast<uint4*>(dst + D / 2 + c + 8) = w2[1];
      }
    }
  }
}

// Host entry of the persistent kernel (gemm_persistent.cu); a.rs_vec replaces rs_x.
void launch_gemm_persistent(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int BN,
                            cudaStream_t st);
int gemm_num_sms();
// Profiling: the next launch's span slot (4 x u64) when span tracing is on, else nullptr.
unsigned long long* next_span(const char* name);

}  // namespace braid
