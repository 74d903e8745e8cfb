// tkv_frag.cuh -- register-level pieces shared by the decode and prefill
// kernels of the paged KIVI format: the compile-time page layout, the
// per-thread loads of key- and value-code words, and the dequantisation of
// codes straight into mma.m16n8k16 fragments.
//
// Fragment correspondence used by both kernels: key_frag() builds the A
// operand of a 16-token x 16-channel key tile (registers {r0, r2} hold the
// thread's row g = token g, {r1, r3} row g + 8), which is also the B operand
// (k = channel, n = token) of an 8-token tile: {r0, r2} for tokens 0-7 and
// {r1, r3} for tokens 8-15.  value_frag() likewise gives the A operand of a
// 16-channel x 16-token V^T tile, which is the B operand (k = token,
// n = channel) of channels 16mb..16mb+7 as {r0, r2} and 16mb+8..16mb+15 as
// {r1, r3}.
#pragma once

#include "tkv_common.cuh"

namespace tkv {

__device__ __forceinline__ int nq_len(int len, int R, int G) {
  int x = len - R;
  return x > 0 ? G * (x / G) : 0;
}

// Channel (relative to the thread's chunk of D/4 channels) that feeds k-slot
// (2*tig + 8*hi + e) of k-block kb, for the canonical row-major key codes.
template <int BITS>
__device__ __forceinline__ constexpr int kchan(int kb, int hi, int e) {
  return BITS == 4 ? 8 * (kb / 2) + 2 * (kb % 2) + hi + 4 * e
                   : 16 * (kb / 4) + 2 * (kb % 4) + hi + 8 * e;
}

// A-fragment registers (R0..R3 = {a0a1},{a2a3},{a4a5},{a6a7}) of k-block KB:
// fp16 keys dequantised exactly as the reference decompress rounds them,
// k = fp16(code * step + zero), from the thread's key-code words of rows g (wg)
// and g+8 (wh) and the per-channel (step, zero) pairs of this key group.
template <int BITS, int KB>
__device__ __forceinline__ void key_frag(const uint32_t* wg, const uint32_t* wh,
                                         const uint32_t (&ks)[2], const uint32_t (&kz)[2],
                                         uint32_t (&r)[4]) {
  if (BITS == 4) {
    constexpr int j = KB / 2;
    if (KB % 2 == 0) {  // nibbles (0,4) -> hi 0, (1,5) -> hi 1
      r[0] = hfma2(code_pair<0x000F000Fu>(wg[j]), ks[0], kz[0]);
      r[1] = hfma2(code_pair<0x000F000Fu>(wh[j]), ks[0], kz[0]);
      r[2] = hfma2(code_pair<0x00F000F0u>(wg[j]), ks[1], kz[1]);
      r[3] = hfma2(code_pair<0x00F000F0u>(wh[j]), ks[1], kz[1]);
    } else {            // nibbles (2,6) -> hi 0, (3,7) -> hi 1
      const uint32_t g8 = wg[j] >> 8, h8 = wh[j] >> 8;
      r[0] = hfma2(code_pair<0x000F000Fu>(g8), ks[0], kz[0]);
      r[1] = hfma2(code_pair<0x000F000Fu>(h8), ks[0], kz[0]);
      r[2] = hfma2(code_pair<0x00F000F0u>(g8), ks[1], kz[1]);
      r[3] = hfma2(code_pair<0x00F000F0u>(h8), ks[1], kz[1]);
    }
  } else {
    // 2-bit codes i and i+8 pair up; kb = 4j + i/2, hi = i%2
    constexpr int j = KB / 4, u = KB % 4;
    const uint32_t g_ = u < 2 ? wg[j] : (wg[j] >> 8);
    const uint32_t h_ = u < 2 ? wh[j] : (wh[j] >> 8);
    constexpr uint32_t m0 = (u % 2 == 0) ? 0x00030003u : 0x00300030u;  // i = 2u (mod 4)
    constexpr uint32_t m1 = (u % 2 == 0) ? 0x000C000Cu : 0x00C000C0u;  // i = 2u+1 (mod 4)
    r[0] = hfma2(code_pair<m0>(g_), ks[0], kz[0]);
    r[1] = hfma2(code_pair<m0>(h_), ks[0], kz[0]);
    r[2] = hfma2(code_pair<m1>(g_), ks[1], kz[1]);
    r[3] = hfma2(code_pair<m1>(h_), ks[1], kz[1]);
  }
}

// A-fragment registers of m-block MB of V^T from the lane's value-code words.
// 4-bit codes: each register pair becomes 64 + c exactly (the nibble is moved
// to mantissa bits 4..7 of 64.0); 2-bit codes: 1 + c/16.  In both cases
// value = kVScale * reg - kVBeta with the constants below.
// 4-bit codes: tokens 0-7 of the page (k-slots of b01) become 1024 + c, tokens
// 8-15 become 64 + c (nibbles OR-ed into the mantissas of 1024.0 and 64.0);
// value = reg - beta with beta = 1024 / 64 for the two token halves.
// 2-bit codes: 1 + c/16 for both halves, value = 16 * reg - 16.
template <int BITS> struct VEnc;
template <> struct VEnc<4> {
  static constexpr float kScale = 1.f, kBetaLo = 1024.f, kBetaHi = 64.f;
};
template <> struct VEnc<2> {
  static constexpr float kScale = 16.f, kBetaLo = 16.f, kBetaHi = 16.f;
};

template <int BITS, int MB>
__device__ __forceinline__ void value_frag(const uint32_t* vw, uint32_t (&r)[4]) {
  if (BITS == 4) {
    const uint32_t w = vw[MB], w8 = w >> 8;
    r[0] = and_or(w, 0x000F000Fu, 0x64006400u);   // nibbles 0,4: rows g,   tokens 2tig, 2tig+1
    r[2] = and_or(w, 0x00F000F0u, 0x54005400u);   // nibbles 1,5: rows g,   tokens +8
    r[1] = and_or(w8, 0x000F000Fu, 0x64006400u);  // nibbles 2,6: rows g+8, tokens 2tig, 2tig+1
    r[3] = and_or(w8, 0x00F000F0u, 0x54005400u);  // nibbles 3,7: rows g+8, tokens +8
  } else {
    const uint32_t w = vw[MB / 2];
    constexpr int base = 4 * (MB % 2);
    r[0] = ext2<6 - 2 * (base + 0)>(w);
    r[2] = ext2<6 - 2 * (base + 1)>(w);
    r[1] = ext2<6 - 2 * (base + 2)>(w);
    r[3] = ext2<6 - 2 * (base + 3)>(w);
  }
}

// ---------------------------------------------------------------------------
// compile-time layout of one paged format (same numbers as tkv_format_init)
// ---------------------------------------------------------------------------
template <int D, int BITS, int G>
struct Fmt {
  static constexpr int NKB = D / 16;             // k-blocks of QK / m-blocks of PV
  static constexpr int CH = D / 4;               // key channels per thread chunk
  static constexpr int RB = D * BITS / 8;        // key-code bytes per token row
  static constexpr int TW = RB / 16;             // key-code words per thread per row
  static constexpr int VWN = D * BITS / 64;      // value-code words per lane
  static constexpr int VW = VWN < 4 ? VWN : 4;   // value-code words per 16-byte vector
  static constexpr int NVG = D > G ? D / G : 1;  // value groups per token
  static constexpr int MB_PER_VG = (D / 16) / NVG;
  static constexpr int CODES = kPage * D * BITS / 8;
  static constexpr int V_CODES_OFF = CODES;
  static constexpr int V_META_OFF = 2 * CODES;
  static constexpr int BODY = 2 * CODES + kPage * NVG * 4;  // page bytes before the key meta
  static constexpr int KMS = D * 4 * kPage / G;              // key-meta slice bytes per page
  static constexpr int PB = (BODY + KMS + 15) / 16 * 16;     // page_bytes
  static constexpr int PPG = G / kPage;                      // pages per key group
  static constexpr int META = D * 4;                         // key meta bytes per group
  static constexpr int NP = PPG >= 2 ? 2 : 1;                // pages per ring stage / softmax step
  static constexpr int RBLK = kPage * D * 2;                 // residual K (or V) block of a chunk
  static constexpr int SB = ((NP * BODY > RBLK ? NP * BODY : RBLK) + 127) / 128 * 128;
  static constexpr int ST = (13312 / SB) < 2 ? 2 : (13312 / SB) > 8 ? 8 : (13312 / SB);  // stages
  static_assert(TW >= 1 && (RB % 16) == 0, "key row split");
  static_assert((KMS % 16) == 0 && (BODY % 16) == 0, "bulk-copy sizes are multiples of 16");
};

template <int D, int BITS, int G>
constexpr int decode_smem_bytes() {
  using F = Fmt<D, BITS, G>;
  return 128 + F::ST * F::SB + 2 * F::META;
}

// Loads the thread's 8 (or fewer) key-code words of rows g and g+8.
template <int D, int BITS>
__device__ __forceinline__ void load_key_words(const uint8_t* kc, int g, int tig,
                                               uint32_t (&wg)[D * BITS / 128],
                                               uint32_t (&wh)[D * BITS / 128]) {
  constexpr int RB = D * BITS / 8, TB = RB / 4;
  if constexpr (TB == 16) {
    const uint4 x = *reinterpret_cast<const uint4*>(kc + g * RB + tig * 16);
    const uint4 y = *reinterpret_cast<const uint4*>(kc + (g + 8) * RB + tig * 16);
    wg[0] = x.x; wg[1] = x.y; wg[2] = x.z; wg[3] = x.w;
    wh[0] = y.x; wh[1] = y.y; wh[2] = y.z; wh[3] = y.w;
  } else if constexpr (TB == 8) {
    const uint2 x = *reinterpret_cast<const uint2*>(kc + g * RB + tig * 8);
    const uint2 y = *reinterpret_cast<const uint2*>(kc + (g + 8) * RB + tig * 8);
    wg[0] = x.x; wg[1] = x.y;
    wh[0] = y.x; wh[1] = y.y;
  } else {
    wg[0] = *reinterpret_cast<const uint32_t*>(kc + g * RB + tig * 4);
    wh[0] = *reinterpret_cast<const uint32_t*>(kc + (g + 8) * RB + tig * 4);
  }
}

template <int D, int BITS>
__device__ __forceinline__ void load_value_words(const uint8_t* vc, int lane,
                                                 uint32_t (&vw)[D * BITS / 64]) {
  constexpr int VWN = D * BITS / 64, VW = VWN < 4 ? VWN : 4;
#pragma unroll
  for (int v = 0; v < VWN / VW; ++v) {
    if constexpr (VW == 4) {
      const uint4 x = *reinterpret_cast<const uint4*>(vc + (v * 32 + lane) * 16);
      vw[4 * v + 0] = x.x; vw[4 * v + 1] = x.y; vw[4 * v + 2] = x.z; vw[4 * v + 3] = x.w;
    } else {
      const uint2 x = *reinterpret_cast<const uint2*>(vc + lane * 8);
      vw[0] = x.x; vw[1] = x.y;
    }
  }
}

// Running maxima are only raised when a tile's maximum exceeds them by more
// than kLazyLog2 (log2 units), so most tiles skip the O rescale; weights are
// then at most 2^kLazyLog2 = 4, which keeps p * step_v inside the f16 range for
// any fp16 value range (step_v <= 131008 / 15).
constexpr float kLazyLog2 = 2.0f;

}  // namespace tkv
