// tkv_stream.cu -- balanced ("stream") paged KIVI decode attention on sm_100a.
//
// The attention of tkv_decode.cu (the megakernel math of
// third_party/custom_kernels/megakernel.cu:267-350 over the KIVI pages, with
// the split-KV log-sum-exp merge of paged_attention_v2.cu:132-170), with the
// work laid out for B200 instead of handed out from a queue.
//
// The work of one call is one axis of units: for every (sequence, kv head)
// pair in order, its quantised pages in steps of NP pages (cost 1 per page)
// and then its fp16 residual chunks of 16 tokens (cost kRcCost each).  With C
// the total cost and n the number of warps, warp w owns the units that start
// in [ceil(w C / n), ceil((w+1) C / n)): every warp gets the same cost, there
// is no work counter to claim from and no tail of uneven items.  Each warp
// streams its range through a ring of ST stages that runs on across pair
// boundaries: the next pair's pages, key meta and q rows are in flight while
// the current pair finishes.  Page bodies and q rows move by 1-D bulk copies
// (cp.async.bulk, no multicast) issued by lane 0; a key group's meta
// [D][step, zero] (one slice in each of its pages) moves by one 16-byte
// cp.async per lane.  The block-table entries of the pages ahead are held one
// per lane (a window of 32 pages, checked against the pool once when loaded).
//
// A pair spread over warps w_lo .. w_hi (the owners of its first and last
// unit) leaves one partial (m, l, o[D]) per q head and warp in slot w + p
// (p = the pair's index; the slots of one pair are consecutive, and w + p is
// unique because warps and pairs are both ordered along the axis).  In the
// fused mode the warp that finishes a pair's last partial merges them into
// out (a pair owned by one warp is written directly); in the partials mode
// stream_merge_kernel does it in a second launch (few pairs with long
// contexts, where one pair spans many warps and a single warp's serial merge
// would be the launch's tail).
//
// Per unit the math is the decode_warp_kernel's: QK^T and PV on mma.m16n8k16
// with the key codes dequantised exactly to fp16(code * step + zero) in
// registers, online softmax in the exp2 domain, per-token value steps folded
// into P and value zero points added once per head.
#include <algorithm>
#include <atomic>

#include "tkv_decode_common.cuh"

namespace tkv {

// cost of a 16-token fp16 residual chunk in page units (a quantised page = 1)
#ifndef TKV_STREAM_RC_COST
#define TKV_STREAM_RC_COST 2
#endif
// fewest cost units per warp: small calls use fewer warps (a warp alone on
// its SM runs a step in about 2 us, so short chains keep small calls short)
#ifndef TKV_STREAM_MIN_COST
#define TKV_STREAM_MIN_COST 8
#endif
// independent warps per CTA, and resident warps per SM the register budget targets
#ifndef TKV_STREAM_WPC
#define TKV_STREAM_WPC 4
#endif
#ifndef TKV_STREAM_WARPS_PER_SM
#define TKV_STREAM_WARPS_PER_SM 12
#endif
#ifndef TKV_STREAM_STAGES
#define TKV_STREAM_STAGES 3
#endif
// most quantised pages per ring stage and softmax step (capped by the pages
// of one key group)
#ifndef TKV_STREAM_PAGES
#define TKV_STREAM_PAGES 2
#endif
// pages between folds of the value-zero correction into the accumulator
// (WarpState::fold): bounds the code offset a long run carries in fp32
#ifndef TKV_STREAM_FOLD_PAGES
#define TKV_STREAM_FOLD_PAGES 16
#endif

constexpr int kRcCost = TKV_STREAM_RC_COST;
constexpr int kMinCost = TKV_STREAM_MIN_COST;
constexpr int kWPC = TKV_STREAM_WPC;
constexpr int kWarpsPerSM = TKV_STREAM_WARPS_PER_SM;
constexpr int kFoldPages = TKV_STREAM_FOLD_PAGES;
// Bound on the warps of one launch used to size the workspace (148 SMs x 16);
// a launch uses min(resident warps, what the workspace's slots allow).
constexpr int kStreamMaxWarps = 148 * 16;
constexpr int kMaxDevices = 64;
static_assert(kWarpsPerSM % kWPC == 0, "whole CTAs per SM");
static_assert(kFoldPages % 2 == 0, "folds fall on step boundaries (1 or 2 pages a step)");

// Stage layout: a quantised step (NP page bodies, then the key-group meta when
// the step starts a group) or one half (K or V block) of a residual chunk.
template <int D, int BITS, int G>
struct SFmt {
  using F = Fmt<D, BITS, G>;
  static constexpr int NP = F::PPG < TKV_STREAM_PAGES ? F::PPG : TKV_STREAM_PAGES;
  static_assert(F::PPG % NP == 0, "steps do not straddle key groups");
  static_assert(NP <= 4, "at most four page copies per stage");
  static constexpr int META_OFF = NP * F::BODY;
  // The key-group meta arrives as MCH chunks of 16 bytes; each thread reads
  // the CH channel words of its tig chunk, so a 16-byte pad after every tig
  // chunk puts the four tig chunks in different banks.
  static constexpr int MCH = F::META / 16;  // 16-byte chunks of the group meta
  static constexpr int TCH = F::CH / 4;     // chunks per tig chunk
  static constexpr int CPS = F::KMS / 16;   // chunks per page's meta slice
  static constexpr int META_PAD = F::META + (MCH / TCH) * 16;
  static constexpr int QSTEP = META_OFF + META_PAD;
  static constexpr int SB = ((QSTEP > F::RBLK ? QSTEP : F::RBLK) + 127) / 128 * 128;
  static constexpr int ST = TKV_STREAM_STAGES;
  static_assert(META_OFF % 16 == 0, "copy destinations are 16-byte aligned");
  static_assert(MCH <= 32, "one 16-byte meta chunk per lane");
};

// Shared memory of one warp: [ring ST x SB][tail][q buffers 2 x grp x D x 2 B].
// Tail: mbarriers [0, ST) stage bodies (one arrival + bulk-copy bytes),
// [ST, 2 ST) stage key meta (32 cp.async arrivals), [2 ST, 2 ST + 2) q
// buffers; the control block at kStreamTailBars mbarrier slots.
constexpr int kStreamTailBars = 16;
constexpr int kStreamTail = 512;
template <int D, int BITS, int G>
constexpr int stream_ring_bytes() {
  return SFmt<D, BITS, G>::ST * SFmt<D, BITS, G>::SB;
}
inline int stream_warp_smem(int ring_bytes, int grp, int D) {
  return ring_bytes + kStreamTail + 2 * grp * D * 2;
}
static_assert(2 * TKV_STREAM_STAGES + 2 <= kStreamTailBars, "barriers fit before the control block");
static_assert(TKV_STREAM_STAGES <= 8, "stage index and meta parities fit the packed counter");

__device__ __forceinline__ int warp_sum(int x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

__device__ __forceinline__ int warp_incl_scan(int x, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  return x;
}

__device__ __forceinline__ long long shfl_ll(long long x, int src) {
  const int lo = __shfl_sync(0xffffffffu, static_cast<int>(x & 0xffffffffLL), src);
  const int hi = __shfl_sync(0xffffffffu, static_cast<int>(x >> 32), src);
  return (static_cast<long long>(hi) << 32) | static_cast<unsigned int>(lo);
}

// Work of one sequence (the same for each of its kv heads): quantised pages
// [pg0, pg0 + npg) of the call's page range, nrc residual chunks after the
// nq quantised tokens.  Returns the cost, or -1 for a length out of range
// (no work; flagged by the pair's owner).
template <int G>
__device__ __forceinline__ int seq_work(const StreamArgs& a, int len, int& npg, int& nrc,
                                        int& pg0, int& nq) {
  npg = nrc = pg0 = nq = 0;
  if (len < 0 || len > a.max_len || static_cast<long long>(len) >
                                        static_cast<long long>(a.max_blocks) * kPage)
    return -1;
  nq = nq_len(len, a.residual, G);
  const int tp = nq / kPage;
  pg0 = min(a.pg_lo, tp);
  npg = min(a.pg_hi, tp) - pg0;
  nrc = a.include_residual ? (len - nq + kPage - 1) / kPage : 0;
  return npg + kRcCost * nrc;
}

// Position on the work axis: pair (b, h) and the data of sequence b.
struct Cursor {
  long long start;  // cost position of the pair's first unit
  int b, h;
  int len, nq, npg, nrc, pg0, cost;
  int bad;          // length out of range
};

template <int G>
__device__ __forceinline__ void cursor_load(const StreamArgs& a, Cursor& c) {
  c.len = __ldg(a.seq_lens + c.b);
  const int x = seq_work<G>(a, c.len, c.npg, c.nrc, c.pg0, c.nq);
  c.bad = x < 0;
  c.cost = x > 0 ? x : 0;
}

// next pair in axis order; false past the last one
template <int G>
__device__ __forceinline__ bool cursor_next(const StreamArgs& a, Cursor& c) {
  c.start += c.cost;
  if (++c.h < a.n_kv_heads) return true;
  c.h = 0;
  if (++c.b >= a.num_seqs) return false;
  cursor_load<G>(a, c);
  return true;
}

// Index of the first unit of a pair whose start offset is >= x: units
// 0 .. npg/NP - 1 are quantised steps (offset NP u), the rest residual chunks
// (offset npg + kRcCost (u - npg/NP)).
template <int NP>
__device__ __forceinline__ int unit_at(long long x, int npg, int nrc) {
  if (x <= 0) return 0;
  if (x <= npg) return static_cast<int>((x + NP - 1) / NP);
  const long long r = (x - npg + kRcCost - 1) / kRcCost;
  return npg / NP + static_cast<int>(r < nrc ? r : nrc);
}

// q of head g from a q buffer as a float (f16 or bf16 bits)
__device__ __forceinline__ float qbuf_val(const uint16_t* qh, int c, bool bf16) {
  const uint16_t x = qh[c];
  return bf16 ? __uint_as_float(static_cast<uint32_t>(x) << 16)
              : __half2float(__ushort_as_half(x));
}

// sums l and the value-zero corrections w over the 8 token rows of the warp
template <int D, int NVG>
__device__ __forceinline__ void state_reduce(WarpState<D, NVG>& st) {
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    float l = st.l[hh];
    l += __shfl_xor_sync(0xffffffffu, l, 4);
    l += __shfl_xor_sync(0xffffffffu, l, 8);
    l += __shfl_xor_sync(0xffffffffu, l, 16);
    st.l[hh] = l;
#pragma unroll
    for (int vg = 0; vg < NVG; ++vg) {
      float w = st.w[vg][hh];
      w += __shfl_xor_sync(0xffffffffu, w, 4);
      w += __shfl_xor_sync(0xffffffffu, w, 8);
      w += __shfl_xor_sync(0xffffffffu, w, 16);
      st.w[vg][hh] = w;
    }
  }
}

// Writes the warp's (reduced) state for the grp q heads: as a partial slot
// (po [grp][D], pml [grp][2]) or, when out != nullptr, normalised into out
// rows orow .. orow + grp - 1 (the arithmetic of a one-slot merge).
template <int D, int NVG>
__device__ __forceinline__ void state_write(const WarpState<D, NVG>& st, int grp, float oscale,
                                            float* po, float* pml, void* out, int out_dtype,
                                            int64_t orow) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
  constexpr int MB_PER_VG = (D / 16) / NVG;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int hd = 2 * tig + hh;
    if (hd >= grp) continue;
    const float inv = st.l[hh] > 0.f ? 1.f / st.l[hh] : 0.f;
#pragma unroll
    for (int mb = 0; mb < D / 16; ++mb) {
      const int vg = mb / MB_PER_VG;
      const float o0 = fmaf(oscale, st.o[mb][hh], st.w[vg][hh]);
      const float o1 = fmaf(oscale, st.o[mb][2 + hh], st.w[vg][hh]);
      const int c0 = 16 * mb + g, c1 = c0 + 8;
      if (out == nullptr) {
        po[hd * D + c0] = o0;
        po[hd * D + c1] = o1;
      } else {
        const int64_t i0 = (orow + hd) * D + c0, i1 = (orow + hd) * D + c1;
        const float v0 = o0 * inv, v1 = o1 * inv;
        if (out_dtype == TKV_F32) {
          static_cast<float*>(out)[i0] = v0;
          static_cast<float*>(out)[i1] = v1;
        } else if (out_dtype == TKV_BF16) {
          static_cast<__nv_bfloat16*>(out)[i0] = __float2bfloat16_rn(v0);
          static_cast<__nv_bfloat16*>(out)[i1] = __float2bfloat16_rn(v1);
        } else {
          static_cast<__half*>(out)[i0] = __float2half_rn(v0);
          static_cast<__half*>(out)[i1] = __float2half_rn(v1);
        }
      }
    }
    if (out == nullptr && g == 0) {
      pml[hd * 2 + 0] = st.m[hh];
      pml[hd * 2 + 1] = st.l[hh];
    }
  }
}

// A work pair of one warp (its unit range [u0, u1)), in the warp's control
// block; row = ring row (0 when the pair has no residual units here).
struct Desc {
  long long start;
  int b, h, len, nq, npg, nrc, pg0, u0, u1, row;
};

// Warp-uniform state touched once per pair, not per unit: kept in shared
// memory so the registers go to the accumulators.
struct Ctl {
  Cursor walk;        // the issue side's position on the axis
  Desc d[2];          // work pair k of the warp in d[k & 1]
  long long S, E, C;  // the warp's range and the total cost
  int nw, last, first, live;
};
static_assert(kStreamTailBars * 8 + sizeof(Ctl) <= kStreamTail, "control block fits the tail");

template <int D, int BITS, int G>
__global__ void __launch_bounds__(32 * kWPC, kWarpsPerSM / kWPC)
    decode_stream_kernel(StreamArgs a) {
  using F = Fmt<D, BITS, G>;
  using SF = SFmt<D, BITS, G>;
  constexpr int NP = SF::NP, NVG = F::NVG, PPG = F::PPG, ST = SF::ST, SB = SF::SB;
  extern __shared__ __align__(128) uint8_t smem_all[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
  const int wid = blockIdx.x * kWPC + warp;
  if (wid >= a.n_warps) return;
  const int qbytes = a.grp * D * 2;
  uint8_t* const ring = smem_all + warp * a.warp_smem;
  uint64_t* const bars = reinterpret_cast<uint64_t*>(ring + ST * SB);
  Ctl& ctl = *reinterpret_cast<Ctl*>(bars + kStreamTailBars);
  uint8_t* const qbuf = ring + ST * SB + kStreamTail;
  const int Hkv = a.n_kv_heads;

  {
    // ---- the axis: total cost C, this warp's range [S, E) ----
    long long cseq = 0;
    for (int b0 = 0; b0 < a.num_seqs; b0 += 32) {
      int c = 0;
      if (b0 + lane < a.num_seqs) {
        int npg, nrc, pg0, nq;
        c = max(0, seq_work<G>(a, __ldg(a.seq_lens + b0 + lane), npg, nrc, pg0, nq));
      }
      cseq += warp_sum(c);
    }
    const long long C = cseq * Hkv;
    const int nw =
        static_cast<int>(min(static_cast<long long>(a.n_warps), max(1LL, C / kMinCost)));
    if (wid >= nw) return;
    const long long S = (wid * C + nw - 1) / nw;
    const long long E = ((wid + 1) * C + nw - 1) / nw;

    // first pair at or after S: the pair holding position S, or a pair with
    // no work placed at a position >= S
    Cursor c0;
    c0.b = a.num_seqs;
    long long carry = 0;
    for (int b0 = 0; b0 < a.num_seqs; b0 += 32) {
      const int b = b0 + lane;
      int c = 0;
      if (b < a.num_seqs) {
        int npg, nrc, pg0, nq;
        c = max(0, seq_work<G>(a, __ldg(a.seq_lens + b), npg, nrc, pg0, nq));
      }
      const int incl = warp_incl_scan(c, lane);
      const long long pre = carry + (incl - c);
      const bool hit = b < a.num_seqs && (c == 0 ? pre * Hkv >= S : (pre + c) * Hkv > S);
      const unsigned int m = __ballot_sync(0xffffffffu, hit);
      if (m) {
        const int src = __ffs(m) - 1;
        const long long pb = shfl_ll(pre, src);
        const int cb = __shfl_sync(0xffffffffu, c, src);
        c0.b = b0 + src;
        c0.h = cb > 0 ? static_cast<int>(max(0LL, S - pb * Hkv) / cb) : 0;
        c0.start = pb * Hkv + static_cast<long long>(c0.h) * cb;
        break;
      }
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (c0.b >= a.num_seqs) return;
    cursor_load<G>(a, c0);
    if (lane == 0) {
      ctl.walk = c0;
      ctl.S = S;
      ctl.E = E;
      ctl.C = C;
      ctl.nw = nw;
      ctl.last = wid == nw - 1;
      ctl.first = 1;
      ctl.live = 1;
      for (int i = 0; i < 2 * ST + 2; ++i) mbar_init(&bars[i], i >= ST && i < 2 * ST ? 32 : 1);
      fence_mbar_init();
    }
    __syncwarp();
  }

  // ---------------- issue side ----------------
  int isu = 0, isu1 = 0;  // next stage unit of the issue pair and its end
  int ik = -1;            // work pairs entered by the issue side
  int pgb = 0;            // the lanes hold block-table entries of pages pgb + lane
  int pid = 0;
  int istg = 0;           // stage the next issue fills
  int nin = 0;            // stages in flight
  int ck = 0;             // work pair the consume side is on
  // consume side's ring position: bits 0-3 stage, bit 4 its phase parity,
  // bit 8 + s the parity of stage s's key-meta barrier
  uint32_t cst = 0;

  // Pairs without work at positions this warp owns: zeros into out (fused)
  // or an empty slot range for the merge kernel, and the length error.
  auto empty_pair = [&](const Cursor& c) {
    const int p = c.b * Hkv + c.h;
    if (c.bad && lane == 0) set_err(a.err, TKV_ERR_BAD_LENGTH);
    if (a.mode == kStreamPartials) {
      if (lane == 0) a.pair_info[p] = make_int2(0, 0);
      return;
    }
    const int64_t base = (static_cast<int64_t>(c.b) * a.num_q_heads + c.h * a.grp) * D;
    for (int i = lane; i < a.grp * D; i += 32) {
      if (a.out_dtype == TKV_F32)
        static_cast<float*>(a.out)[base + i] = 0.f;
      else if (a.out_dtype == TKV_BF16)
        static_cast<__nv_bfloat16*>(a.out)[base + i] = __float2bfloat16_rn(0.f);
      else
        static_cast<__half*>(a.out)[base + i] = __float2half_rn(0.f);
    }
  };

  // Walks the axis to the next pair with units of this warp (the walk's
  // current pair on the first call), handling the empty pairs passed on the
  // way; writes the pair to ctl.d[(ik + 1) & 1].
  auto seek = [&]() -> bool {
    Cursor c = ctl.walk;
    bool first = ctl.first != 0;
    const long long S = ctl.S, E = ctl.E, C = ctl.C;
    const bool last = ctl.last != 0;
    bool found = false;
    int u0 = 0, u1 = 0;
    for (;;) {
      if (!first && !cursor_next<G>(a, c)) break;
      first = false;
      if (!(c.start < E || (last && c.start == C))) break;
      if (c.cost == 0) {
        if (c.start >= S) empty_pair(c);
        continue;
      }
      u0 = unit_at<NP>(S - c.start, c.npg, c.nrc);
      u1 = unit_at<NP>(E - c.start, c.npg, c.nrc);
      if (u0 < u1) {
        found = true;
        break;
      }
    }
    int row = 0;
    if (found && u1 > c.npg / NP) {  // residual units: the sequence's ring row
      row = a.seq_slots ? __ldg(a.seq_slots + c.b) : c.b;
      if (row < 0 || row >= a.max_seqs) {
        if (lane == 0) set_err(a.err, TKV_ERR_BAD_SLOT);
        row = 0;  // read in bounds; the sequence's output is not meaningful
      }
    }
    __syncwarp();
    if (lane == 0) {
      ctl.walk = c;
      ctl.first = 0;
      if (found) {
        Desc& d = ctl.d[(ik + 1) & 1];
        d.start = c.start;
        d.b = c.b;
        d.h = c.h;
        d.len = c.len;
        d.nq = c.nq;
        d.npg = c.npg;
        d.nrc = c.nrc;
        d.pg0 = c.pg0;
        d.u0 = u0;
        d.u1 = u1;
        d.row = row;
      }
    }
    __syncwarp();
    return found;
  };

  // fills stage istg with stage unit isu of the issue pair
  auto issue_one = [&]() {
    const Desc& d = ctl.d[ik & 1];
    const uint64_t pol = l2_evict_first_policy();  // pages and ring rows: read once
    uint8_t* dst = ring + istg * SB;
    uint64_t* bar = &bars[istg];
    const int nst = d.npg / NP;
    if (isu < nst) {
      const int pg = d.pg0 + isu * NP;  // page index in the sequence
      const int gs = pg - pg % PPG;     // first page of its key group
      if (gs < pgb || gs + PPG > pgb + 32) {
        // next 32 block-table entries, checked against the pool once
        pgb = gs;
        const int e = pgb + lane;
        pid = e < d.pg0 + d.npg ? __ldg(a.block_tables + static_cast<int64_t>(d.b) * a.max_blocks + e)
                                : 0;
        const bool bad = pid < 0 || pid >= a.num_pages;
        if (__any_sync(0xffffffffu, bad) && lane == 0) set_err(a.err, TKV_ERR_BAD_PAGE);
        if (bad) pid = 0;  // read in bounds; the sequence's output is not meaningful
      }
      const int p0 = __shfl_sync(0xffffffffu, pid, pg - pgb);
      const int p1 = NP > 1 ? __shfl_sync(0xffffffffu, pid, pg - pgb + 1) : p0;
      const int p2 = NP > 2 ? __shfl_sync(0xffffffffu, pid, pg - pgb + 2) : p0;
      const int p3 = NP > 3 ? __shfl_sync(0xffffffffu, pid, pg - pgb + 3) : p0;
      const uint8_t* ph = a.pool + static_cast<int64_t>(d.h) * F::PB;
      const int64_t ps = static_cast<int64_t>(Hkv) * F::PB;
      if (lane == 0) {
        mbar_arrive_expect_tx(bar, NP * F::BODY);
        bulk_g2s_hint(dst, ph + p0 * ps, F::BODY, bar, pol);
        if (NP > 1) bulk_g2s_hint(dst + F::BODY, ph + p1 * ps, F::BODY, bar, pol);
        if (NP > 2) bulk_g2s_hint(dst + 2 * F::BODY, ph + p2 * ps, F::BODY, bar, pol);
        if (NP > 3) bulk_g2s_hint(dst + 3 * F::BODY, ph + p3 * ps, F::BODY, bar, pol);
      }
      if (pg == gs || isu == d.u0) {
        // the group's key meta: lane l brings chunk l of [D][step, zero]
        const int mc = lane < SF::MCH ? lane : 0;
        const int pm = __shfl_sync(0xffffffffu, pid, gs - pgb + mc / SF::CPS);
        if (lane < SF::MCH)
          cp_async16_hint(dst + SF::META_OFF + (mc + mc / SF::TCH) * 16,
                          ph + pm * ps + F::BODY + (mc % SF::CPS) * 16, pol);
        cp_async_mbar_arrive(&bars[ST + istg]);
      }
    } else if (lane == 0) {
      const int r = isu - nst;  // 2 * chunk + (0: K block, 1: V block)
      const int chunk = ((d.nq + (r >> 1) * kPage) % a.ring_cap) / kPage;
      const uint8_t* src =
          reinterpret_cast<const uint8_t*>(a.ring) +
          (((static_cast<int64_t>(d.row) * Hkv + d.h) * (a.ring_cap / kPage) + chunk) * 2 +
           (r & 1)) *
              F::RBLK;
      mbar_arrive_expect_tx(bar, F::RBLK);
      bulk_g2s_hint(dst, src, F::RBLK, bar, pol);
    }
    __syncwarp();
    ++isu;
    ++nin;
    istg = istg + 1 == ST ? 0 : istg + 1;
  };

  // keeps ST stages in flight; enters the next work pair once its q buffer is free
  auto top_up = [&]() {
    while (nin < ST) {
      if (isu == isu1) {
        if (ik + 1 > ck + 1 || !ctl.live) return;  // its q buffer is still read, or done
        if (!seek()) {
          if (lane == 0) ctl.live = 0;
          __syncwarp();
          return;
        }
        ++ik;
        const Desc& d = ctl.d[ik & 1];
        const int nst = d.npg / NP;
        isu = d.u0 < nst ? d.u0 : nst + 2 * (d.u0 - nst);
        isu1 = d.u1 < nst ? d.u1 : nst + 2 * (d.u1 - nst);
        pgb = -(1 << 30);  // the held block-table entries belong to the last pair
        if (lane == 0) {
          uint64_t* qb = &bars[2 * ST + (ik & 1)];
          mbar_arrive_expect_tx(qb, qbytes);
          bulk_g2s(qbuf + (ik & 1) * qbytes,
                   static_cast<const uint8_t*>(a.q) +
                       (static_cast<int64_t>(d.b) * a.num_q_heads + d.h * a.grp) * D * 2,
                   qbytes, qb);
        }
        __syncwarp();
      }
      issue_one();
    }
  };

  top_up();
  if (ik < 0) return;  // no work pair here (nothing in flight)

  // ---------------- consume side ----------------
  WarpState<D, NVG> st;
  uint32_t bq[F::NKB][2];
  uint32_t ks[F::NKB][2], kz[F::NKB][2];
  bool alive = true;
  // next stage of the consume side (its phase flips on wrap-around)
  auto advance = [&]() {
    const uint32_t s = cst & 15u;
    cst = s + 1 == ST ? ((cst & ~31u) | ((cst & 16u) ^ 16u)) : cst + 1;
    --nin;
  };

  for (;;) {
    // ---- enter work pair ck: its q rows ----
    const Desc& d = ctl.d[ck & 1];
    const int nst = d.npg / NP, cu0 = d.u0, cu1 = d.u1;
    if (!mbar_wait_fast(&bars[2 * ST + (ck & 1)], (ck >> 1) & 1, a.err)) {
      alive = false;
      break;
    }
    const uint16_t* qh = reinterpret_cast<const uint16_t*>(qbuf + (ck & 1) * qbytes) + g * D;
    auto q_quant = [&]() {  // q of head g as exact f16 in this thread's key-channel order
      const bool hok = g < a.grp, qbf = a.q_bf16 != 0;
#pragma unroll
      for (int kb = 0; kb < F::NKB; ++kb)
#pragma unroll
        for (int hi = 0; hi < 2; ++hi) {
          const int c0 = tig * F::CH + kchan<BITS>(kb, hi, 0);
          const int c1 = tig * F::CH + kchan<BITS>(kb, hi, 1);
          bq[kb][hi] = hok ? pack_h2(qbuf_val(qh, c0, qbf), qbuf_val(qh, c1, qbf)) : 0u;
        }
    };
    auto q_resid = [&]() {  // q of head g in the canonical channel order of the ring
      const bool hok = g < a.grp, qbf = a.q_bf16 != 0;
#pragma unroll
      for (int kb = 0; kb < F::NKB; ++kb)
#pragma unroll
        for (int hi = 0; hi < 2; ++hi) {
          const int c = 16 * kb + 2 * tig + 8 * hi;
          bq[kb][hi] = hok ? pack_h2(qbuf_val(qh, c, qbf), qbuf_val(qh, c + 1, qbf)) : 0u;
        }
    };
    if (cu0 < nst)
      q_quant();
    else
      q_resid();
    st.init();

    for (int u = cu0; u < cu1; ++u) {
      if (u < nst) {
        // =================== quantised step: NP pages ===================
        const int cstg = static_cast<int>(cst & 15u);
        if (!mbar_wait_fast(&bars[cstg], (cst >> 4) & 1u, a.err)) {
          alive = false;
          break;
        }
        const uint8_t* sbase = ring + cstg * SB;
        // page range starts (0 or a multiple of 32 pages) are key-group aligned
        if ((u * NP) % PPG == 0 || u == cu0) {
          if (!mbar_wait_fast(&bars[ST + cstg], (cst >> (8 + cstg)) & 1u, a.err)) {
            alive = false;
            break;
          }
          cst ^= 1u << (8 + cstg);
          // this thread's CH channel words (its tig chunk), then the
          // per-channel (step, zero) pairs of the key group as f16x2
          uint32_t mw[F::CH];
          const uint4* mv =
              reinterpret_cast<const uint4*>(sbase + SF::META_OFF) + tig * (SF::TCH + 1);
#pragma unroll
          for (int j = 0; j < SF::TCH; ++j) {
            const uint4 x = mv[j];
            mw[4 * j] = x.x;
            mw[4 * j + 1] = x.y;
            mw[4 * j + 2] = x.z;
            mw[4 * j + 3] = x.w;
          }
#pragma unroll
          for (int kb = 0; kb < F::NKB; ++kb)
#pragma unroll
            for (int hi = 0; hi < 2; ++hi) {
              const uint32_t m0 = mw[kchan<BITS>(kb, hi, 0)];
              const uint32_t m1 = mw[kchan<BITS>(kb, hi, 1)];
              ks[kb][hi] = __byte_perm(m0, m1, 0x5410);
              kz[kb][hi] = __byte_perm(m0, m1, 0x7632);
            }
        }
        // ---- S^T = K Q^T for NP pages (independent MMA chains); columns of
        //      padded heads (>= grp) see q = 0 and are never written ----
        float sc[NP][4];
#pragma unroll
        for (int p = 0; p < NP; ++p) {
          uint32_t wg[F::TW], wh[F::TW];
          load_key_words<D, BITS>(sbase + p * F::BODY, g, tig, wg, wh);
          sc[p][0] = sc[p][1] = sc[p][2] = sc[p][3] = 0.f;
#pragma unroll
          for (int kb = 0; kb < F::NKB; ++kb) {
            uint32_t r[4];
            switch (kb) {
#define TKV_KF(K)                                                                              \
  case K:                                                                                      \
    key_frag<BITS, (K < F::NKB ? K : 0)>(wg, wh, ks[K < F::NKB ? K : 0], kz[K < F::NKB ? K : 0], \
                                         r);                                                   \
    break;
              TKV_KF(0) TKV_KF(1) TKV_KF(2) TKV_KF(3) TKV_KF(4) TKV_KF(5) TKV_KF(6) TKV_KF(7)
#undef TKV_KF
            }
            mma16816(sc[p], r[0], r[1], r[2], r[3], bq[kb][0], bq[kb][1]);
          }
        }
        softmax_update<D, NVG, NP>(st, sc, a.alpha);
        // ---- O^T += V^T P'^T, P' = p * step_v (per token) ----
#pragma unroll
        for (int p = 0; p < NP; ++p) {
          const uint8_t* pgb_ = sbase + p * F::BODY;
          uint32_t vw[F::VWN];
          load_value_words<D, BITS>(pgb_ + F::V_CODES_OFF, lane, vw);
          const uint32_t* vm = reinterpret_cast<const uint32_t*>(pgb_ + F::V_META_OFF);
#pragma unroll
          for (int vg = 0; vg < NVG; ++vg) {
            const float2 sza = unpack_h2(vm[g * NVG + vg]);        // token g:   (step, zero)
            const float2 szb = unpack_h2(vm[(g + 8) * NVG + vg]);  // token g+8
            const uint32_t h2a = pack_h2(sc[p][0] * sza.x, sc[p][1] * sza.x);
            const uint32_t h2b = pack_h2(sc[p][2] * szb.x, sc[p][3] * szb.x);
            const float2 ra = unpack_h2(h2a), rb = unpack_h2(h2b);
            constexpr float blo = VEnc<BITS>::kBetaLo, bhi = VEnc<BITS>::kBetaHi;
            st.w[vg][0] +=
                fmaf(sc[p][0], sza.y, fmaf(sc[p][2], szb.y, -(blo * ra.x + bhi * rb.x)));
            st.w[vg][1] +=
                fmaf(sc[p][1], sza.y, fmaf(sc[p][3], szb.y, -(blo * ra.y + bhi * rb.y)));
            uint32_t b01, b23;
            p_to_bfrag(h2a, h2b, lane, b01, b23);
#pragma unroll
            for (int k = 0; k < F::MB_PER_VG; ++k) {
              const int mb = vg * F::MB_PER_VG + k;
              uint32_t r[4];
              switch (mb) {
#define TKV_VF(M)                                  \
  case M:                                          \
    value_frag<BITS, (M < D / 16 ? M : 0)>(vw, r); \
    break;
                TKV_VF(0) TKV_VF(1) TKV_VF(2) TKV_VF(3) TKV_VF(4) TKV_VF(5) TKV_VF(6) TKV_VF(7)
#undef TKV_VF
              }
              mma16816(st.o[mb], r[0], r[1], r[2], r[3], b01, b23);
            }
          }
        }
        if (((u + 1) * NP) % kFoldPages == 0) st.fold(1.f / VEnc<BITS>::kScale);
        __syncwarp();
        advance();
      } else {
        // =================== fp16 residual chunk: K block, V block ===================
        if (u == nst && cu0 < nst) q_resid();  // the pair's quantised steps came first
        // a stage whose wait gave up stays in flight: the drain below waits for it
        const int sk = static_cast<int>(cst & 15u);
        if (!mbar_wait_fast(&bars[sk], (cst >> 4) & 1u, a.err)) {
          alive = false;
          break;
        }
        advance();
        const int sv = static_cast<int>(cst & 15u);
        if (!mbar_wait_fast(&bars[sv], (cst >> 4) & 1u, a.err)) {
          alive = false;
          break;
        }
        const int tb = d.nq + (u - nst) * kPage;
        const int len = d.len;
        const bool vg0 = tb + g < len, vg8 = tb + g + 8 < len;
        const bool hv0 = 2 * tig < a.grp, hv1 = 2 * tig + 1 < a.grp;
        float sc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
        float(&s)[4] = sc[0];
        const uint8_t* ckb = ring + sk * SB;
#pragma unroll
        for (int kb = 0; kb < F::NKB; ++kb) {
          const uint4 x = *reinterpret_cast<const uint4*>(ckb + (kb * 32 + lane) * 16);
          mma16816(s, x.x, x.y, x.z, x.w, bq[kb][0], bq[kb][1]);
        }
        s[0] = (hv0 && vg0) ? s[0] : -INFINITY;
        s[1] = (hv1 && vg0) ? s[1] : -INFINITY;
        s[2] = (hv0 && vg8) ? s[2] : -INFINITY;
        s[3] = (hv1 && vg8) ? s[3] : -INFINITY;
        softmax_update<D, NVG, 1>(st, sc, a.alpha);
        // fp16 values enter O^T unscaled; the quantised steps' O^T is multiplied
        // by VEnc::kScale at the end, so the weights are divided by it here
        constexpr float kInv = 1.f / VEnc<BITS>::kScale;
        uint32_t b01, b23;
        p_to_bfrag(pack_h2(s[0] * kInv, s[1] * kInv), pack_h2(s[2] * kInv, s[3] * kInv), lane,
                   b01, b23);
        // zero the V^T columns of tokens past the end (stale ring slots)
        const int t0 = tb + 2 * tig;
        const uint32_t m01 = (t0 < len ? 0x0000ffffu : 0u) | (t0 + 1 < len ? 0xffff0000u : 0u);
        const uint32_t m23 =
            (t0 + 8 < len ? 0x0000ffffu : 0u) | (t0 + 9 < len ? 0xffff0000u : 0u);
        const uint8_t* cvb = ring + sv * SB;
#pragma unroll
        for (int mb = 0; mb < D / 16; ++mb) {
          const uint4 x = *reinterpret_cast<const uint4*>(cvb + (mb * 32 + lane) * 16);
          mma16816(st.o[mb], x.x & m01, x.y & m01, x.z & m23, x.w & m23, b01, b23);
        }
        __syncwarp();
        advance();
      }
      top_up();
    }
    if (!alive) break;

    // ---- the pair's partial, its merge ----
    state_reduce<D, NVG>(st);
    {
      const long long C = ctl.C, start = d.start;
      const int nw = ctl.nw;
      const long long lastu =
          start + (d.nrc > 0 ? d.npg + static_cast<long long>(d.nrc - 1) * kRcCost : d.npg - NP);
      const int wlo = static_cast<int>(start * nw / C);
      const int whi = static_cast<int>(lastu * nw / C);
      const int cnt = whi - wlo + 1;
      const int p = d.b * Hkv + d.h;
      const int64_t orow = static_cast<int64_t>(d.b) * a.num_q_heads + d.h * a.grp;
      constexpr float oscale = VEnc<BITS>::kScale;
      if (a.mode == kStreamFused && cnt == 1) {
        state_write<D, NVG>(st, a.grp, oscale, nullptr, nullptr, a.out, a.out_dtype, orow);
      } else {
        const int me = blockIdx.x * kWPC + (threadIdx.x >> 5);  // this warp's index
        const int64_t slot = static_cast<int64_t>(me) + p;
        state_write<D, NVG>(st, a.grp, oscale, a.part_o + slot * a.grp * D,
                            a.part_ml + slot * a.grp * 2, nullptr, 0, 0);
        if (a.mode == kStreamPartials) {
          if (me == wlo && lane == 0) a.pair_info[p] = make_int2(wlo + p, cnt);
        } else {
          __syncwarp();
          __threadfence();  // publish this warp's partial before counting it
          unsigned int old = 0;
          if (lane == 0) old = atomicAdd(&a.pair_count[p], 1u);
          old = __shfl_sync(0xffffffffu, old, 0);
          if (old == static_cast<unsigned int>(cnt - 1)) {
            __threadfence();  // every partial of the pair is visible now
            if (lane == 0) a.pair_count[p] = 0u;
            merge_heads<4>(a.part_ml, a.part_o, cnt, cnt, cnt, a.grp,
                           static_cast<int64_t>(wlo + p) * a.grp, a.grp, D, a.out, a.out_dtype,
                           lane, orow);
          }
        }
      }
    }

    // ---- next work pair ----
    top_up();
    if (ik <= ck) break;
    ++ck;
  }

  if (!alive) {
    // A bounded wait gave up (TKV_ERR_TIMEOUT is set): stop, but first let the
    // copies this warp still has in flight land, each wait bounded again.
    for (int i = 0; i < nin; ++i) {
      uint32_t c = cst;
      for (int k = 0; k < i; ++k) {
        const uint32_t s = c & 15u;
        c = s + 1 == ST ? ((c & ~31u) | ((c & 16u) ^ 16u)) : c + 1;
      }
      mbar_wait(&bars[c & 15u], (c >> 4) & 1u, nullptr);
    }
    cp_async_wait_all();  // the key-meta copies
    // q copies: the current pair's (a completed phase returns at once) and the next one's
    for (int k = ck; k <= ik; ++k) mbar_wait(&bars[2 * ST + (k & 1)], (k >> 1) & 1, nullptr);
  }
}

// ---------------------------------------------------------------------------
// merge of the partials mode: one CTA of kStreamMergeWarps warps per (q head,
// sequence); warp w merges a block of the pair's slots (merge_heads with
// RED), then the warps' results are combined in shared memory with the same
// log-sum-exp rule.  out_ml != nullptr: the unnormalised (M, L) to out_ml and
// O to out (f32, the tkv_paged_decode_range output); pub.world > 0: the same
// unnormalised row into this GPU's slot on every GPU of the exchange, then
// the flag (tkv_exchange_decode_range); else O / L to out.
// ---------------------------------------------------------------------------
#ifndef TKV_STREAM_MERGE_WARPS
#define TKV_STREAM_MERGE_WARPS 8
#endif
constexpr int kStreamMergeWarps = TKV_STREAM_MERGE_WARPS;

__global__ void __launch_bounds__(32 * kStreamMergeWarps)
    stream_merge_kernel(const int2* __restrict__ pair_info, const float* __restrict__ part_ml,
                        const float* __restrict__ part_o, int num_q_heads, int grp, int D,
                        void* __restrict__ out, int out_dtype, float* __restrict__ out_ml,
                        ExPub pub) {
  __shared__ float s_ml[kStreamMergeWarps][2];
  const bool publish = pub.world > 0;
  const uint32_t step = publish ? *reinterpret_cast<volatile uint32_t*>(pub.state) : 0u;
  __shared__ float s_o[kStreamMergeWarps][128];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hq = blockIdx.x, b = blockIdx.y;
  const int hkv = num_q_heads / grp;
  const int p = b * hkv + hq / grp, j = hq % grp;
  const int2 info = pair_info[p];
  const int per = (info.y + kStreamMergeWarps - 1) / kStreamMergeWarps;
  const int s0 = min(info.y, warp * per), cnt = min(info.y, s0 + per) - s0;
  if (cnt > 0) {
    const int64_t first = static_cast<int64_t>(info.x) + s0;
    merge_heads<1, true>(part_ml + first * grp * 2, part_o + first * grp * D, cnt, cnt, cnt, grp,
                         j, 1, D, &s_o[warp][0], TKV_F32, lane, 0, &s_ml[warp][0]);
  } else if (lane == 0) {
    s_ml[warp][0] = -INFINITY;
    s_ml[warp][1] = 0.f;
  }
  __syncthreads();
  float M = -INFINITY;
  for (int w = 0; w < kStreamMergeWarps; ++w) M = fmaxf(M, s_ml[w][0]);
  float L = 0.f;
  for (int w = 0; w < kStreamMergeWarps; ++w) {
    const float m = s_ml[w][0];
    if (m != -INFINITY) L = fmaf(s_ml[w][1], fast_exp2(m - M), L);
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  const int64_t i0 = static_cast<int64_t>(b) * num_q_heads + hq;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float acc = 0.f;
    for (int w = 0; w < kStreamMergeWarps; ++w) {
      const float m = s_ml[w][0];
      if (m != -INFINITY) acc = fmaf(s_o[w][c], fast_exp2(m - M), acc);
    }
    const int64_t oi = i0 * D + c;
    if (publish) {
      ex_store_row(pub, step, i0, c, acc);
    } else if (out_ml) {
      static_cast<float*>(out)[oi] = acc;
    } else {
      const float v = acc * inv;
      if (out_dtype == TKV_F32)
        static_cast<float*>(out)[oi] = v;
      else if (out_dtype == TKV_BF16)
        static_cast<__nv_bfloat16*>(out)[oi] = __float2bfloat16_rn(v);
      else
        static_cast<__half*>(out)[oi] = __float2half_rn(v);
    }
  }
  if (publish) {
    if (threadIdx.x == 0) ex_store_ml(pub, step, i0, M, L);
    ex_signal(pub, step);
  } else if (out_ml && threadIdx.x == 0) {
    out_ml[i0 * 2 + 0] = M;
    out_ml[i0 * 2 + 1] = L;
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

size_t round256(size_t x) { return (x + 255) / 256 * 256; }

// [256 B reserved][pair counters][pair info][part_ml][part_o]; rows = num_seqs
// * num_q_heads bounds the pairs
size_t header_bytes(int num_seqs, int num_q_heads) {
  const size_t rows = static_cast<size_t>(num_seqs) * static_cast<size_t>(num_q_heads);
  return 256 + round256(rows * 4) + round256(rows * 8);
}

// resident warps of one kernel instantiation on the current device (SMs x
// CTAs per SM x warps per CTA) for this q-head group, cached per device
template <int D, int BITS, int G>
int resident_warps(int grp, int smem) {
  static std::atomic<int> cache[kMaxDevices][9];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  const bool cached = dev >= 0 && dev < kMaxDevices && grp >= 1 && grp <= 8;
  if (cached) {
    const int v = cache[dev][grp].load(std::memory_order_relaxed);
    if (v > 0) return v;
  }
  int sms = 0, per_sm = 0;
  const int smem_max = kWPC * stream_warp_smem(stream_ring_bytes<D, BITS, G>(), 8, D);
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaFuncSetAttribute(decode_stream_kernel<D, BITS, G>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_stream_kernel<D, BITS, G>,
                                                    32 * kWPC, smem) != cudaSuccess ||
      per_sm <= 0)
    return -1;
  const int v = sms * per_sm * kWPC;
  if (cached) cache[dev][grp].store(v, std::memory_order_relaxed);
  return v;
}

template <int D, int BITS, int G>
int launch_t(StreamArgs a, cudaStream_t stream) {
  a.warp_smem = stream_warp_smem(stream_ring_bytes<D, BITS, G>(), a.grp, D);
  const int smem = kWPC * a.warp_smem;
  const int resident = resident_warps<D, BITS, G>(a.grp, smem);
  if (resident <= 0) return TKV_BACKEND_ERROR;
  a.n_warps = std::min(a.n_warps, resident);
  const int grid = (a.n_warps + kWPC - 1) / kWPC;
  decode_stream_kernel<D, BITS, G><<<grid, 32 * kWPC, smem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

template <int D, int BITS>
int launch_g(const StreamArgs& a, int group, cudaStream_t stream) {
  switch (group) {
    case 16: return launch_t<D, BITS, 16>(a, stream);
    case 32: return launch_t<D, BITS, 32>(a, stream);
    case 64: return launch_t<D, BITS, 64>(a, stream);
    case 128: return launch_t<D, BITS, 128>(a, stream);
  }
  return TKV_NOT_IMPLEMENTED;
}

}  // namespace

size_t stream_workspace_bytes(int num_seqs, int num_q_heads, int head_dim) {
  const size_t rows = static_cast<size_t>(num_seqs) * static_cast<size_t>(num_q_heads);
  const size_t slot_rows =
      static_cast<size_t>(kStreamMaxWarps) * static_cast<size_t>(std::min(8, num_q_heads)) +
      rows;
  return header_bytes(num_seqs, num_q_heads) +
         slot_rows * (static_cast<size_t>(head_dim) + 2) * sizeof(float);
}

// The fused merge runs in the warp that finishes a pair's last part and reads
// the pair's partial slots one after another; with W resident warps and P
// (sequence, kv head) pairs a pair spans about W / P warps.  Past
// kMaxFusedSpan slots per pair the slot-parallel merge kernel (a second
// launch) is faster: measured on config 2's rank shares, 64 pairs take 28.9 us
// with it and 33.4 us fused, 128 pairs 43.2 us with it and 39.9 us fused.
constexpr int kMaxFusedSpan = 16;

int stream_decode_launches(int num_seqs, int num_kv_heads) {
  static std::atomic<int> warps[kMaxDevices];  // SMs x kWarpsPerSM, per device
  int dev = 0, w = kStreamMaxWarps;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices) {
    w = warps[dev].load(std::memory_order_relaxed);
    if (w <= 0) {
      int sms = 0;
      w = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && sms > 0
              ? sms * kWarpsPerSM
              : kStreamMaxWarps;
      warps[dev].store(w, std::memory_order_relaxed);
    }
  }
  const long long pairs = static_cast<long long>(num_seqs) * num_kv_heads;
  return pairs * kMaxFusedSpan < w ? 2 : 1;
}

int launch_stream_decode(StreamArgs a, int head_dim, int bits, int group, void* workspace,
                         size_t workspace_bytes, float* out_ml, cudaStream_t stream,
                         const ExPub* pub) {
  const size_t hdr = header_bytes(a.num_seqs, a.num_q_heads);
  const size_t slot_bytes = static_cast<size_t>(a.grp) * (head_dim + 2) * sizeof(float);
  if (workspace_bytes < hdr + slot_bytes) return TKV_INVALID_ARGUMENT;
  const long long slots = static_cast<long long>((workspace_bytes - hdr) / slot_bytes);
  const long long pairs = static_cast<long long>(a.num_seqs) * a.n_kv_heads;
  const long long max_warps = slots - pairs + 1;  // slots w + p, w < warps, p < pairs
  if (max_warps < 1) return TKV_INVALID_ARGUMENT;
  a.n_warps = static_cast<int>(std::min<long long>(max_warps, kStreamMaxWarps));
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t rows = static_cast<size_t>(a.num_seqs) * a.num_q_heads;
  a.pair_count = reinterpret_cast<unsigned int*>(ws + 256);
  a.pair_info = reinterpret_cast<int2*>(ws + 256 + round256(rows * 4));
  a.part_ml = reinterpret_cast<float*>(ws + hdr);
  a.part_o = a.part_ml + static_cast<size_t>(slots) * a.grp * 2;
  int st = TKV_NOT_IMPLEMENTED;
  if (head_dim == 128)
    st = bits == 4 ? launch_g<128, 4>(a, group, stream) : launch_g<128, 2>(a, group, stream);
  else if (head_dim == 64)
    st = bits == 4 ? launch_g<64, 4>(a, group, stream) : launch_g<64, 2>(a, group, stream);
  if (st != TKV_OK || a.mode != kStreamPartials) return st;
  dim3 grid(a.num_q_heads, a.num_seqs);
  stream_merge_kernel<<<grid, 32 * kStreamMergeWarps, 0, stream>>>(
      a.pair_info, a.part_ml, a.part_o, a.num_q_heads, a.grp, head_dim, a.out,
      out_ml ? TKV_F32 : a.out_dtype, out_ml, pub ? *pub : ExPub{});
  return cudaGetLastError() == cudaSuccess ? TKV_OK : TKV_BACKEND_ERROR;
}

}  // namespace tkv
