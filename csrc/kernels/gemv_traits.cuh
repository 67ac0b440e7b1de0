// Per-type "part" traits for the dp4a quantized GEMV (decode, 1..8 tokens).
//
// A part is 32 weights of one row.  Lane l of a warp owns parts l, l+32, l+64, ... of the row, so
// a warp's 32 loads of a part-plane are one contiguous 512-byte span (fully coalesced) and, because
// 32 is a multiple of 8, a lane's position inside a 256-weight super-block is the same for every
// part it visits.  Activations are int8 with one (scale, scale*sum) pair per 32 values (ActQ8).
#pragma once
#include "common.cuh"
#include "qweight.cuh"
#include "qtile.cuh"

namespace barq {

BARQ_DEV int4 ld_x16(const int8_t* p) { return *reinterpret_cast<const int4*>(p); }

BARQ_DEV int dot16(int4 w, int4 x) {
  int s = dp4a(w.x, x.x, 0);
  s = dp4a(w.y, x.y, s);
  s = dp4a(w.z, x.z, s);
  return dp4a(w.w, x.w, s);
}

// Integer dot of 32 weights (w0: elements 0-15, w1: 16-31) with the activation at xq; with the
// two-term activation the residual codes ql (step d/256) fold in as 256 * dot(w, q) + dot(w, ql).
template <bool X2>
BARQ_DEV int dot32x(int4 w0, int4 w1, const int8_t* xq, const int8_t* xl) {
  int s = dot16(w0, ld_x16(xq)) + dot16(w1, ld_x16(xq + 16));
  if (X2) s = (s << 8) + dot16(w0, ld_x16(xl)) + dot16(w1, ld_x16(xl + 16));
  return s;
}
template <bool X2>
BARQ_DEV int dot16x(int4 w, const int8_t* xq, const int8_t* xl) {
  int s = dot16(w, ld_x16(xq));
  if (X2) s = (s << 8) + dot16(w, ld_x16(xl));
  return s;
}

BARQ_DEV int4 nib_lo(int4 q) {
  return make_int4(q.x & 0x0F0F0F0F, q.y & 0x0F0F0F0F, q.z & 0x0F0F0F0F, q.w & 0x0F0F0F0F);
}
BARQ_DEV int4 nib_hi(int4 q) {
  return make_int4((q.x >> 4) & 0x0F0F0F0F, (q.y >> 4) & 0x0F0F0F0F, (q.z >> 4) & 0x0F0F0F0F,
                   (q.w >> 4) & 0x0F0F0F0F);
}
BARQ_DEV int4 vsub4(int4 q, int c) {
  return make_int4(__vsub4(q.x, c), __vsub4(q.y, c), __vsub4(q.z, c), __vsub4(q.w, c));
}

// 4-bit code -> signed int8 through a 16-entry byte table (IQ4_NL codebook), four codes per word.
// The 16 table bytes live in t0..t3; PRMT selects bytes 0-7 of a register pair, so the low and
// high halves of the table are looked up separately and merged by each code's bit 3.
BARQ_DEV int lut16(int codes /* 4 bytes, each 0..15 */, int t0, int t1, int t2, int t3) {
  uint32_t c = (uint32_t)codes;
  uint32_t n = (c | (c >> 4));
  uint32_t sel = (n & 0xFFu) | ((n >> 8) & 0xFF00u);  // code_i in nibble i
  uint32_t lo = __byte_perm(t0, t1, sel & 0x7777u);
  uint32_t hi = __byte_perm(t2, t3, sel & 0x7777u);
  uint32_t pick = 0x3210u | ((sel & 0x8888u) >> 1);
  return (int)__byte_perm(lo, hi, pick);
}

// Unpack 6-bit (scale, min) number `is` (0..7) of the 12-byte K-quant scale field held in three
// little-endian words (bytes 0-3, 4-7, 8-11).  Register-only: runtime shifts, no indexed arrays.
BARQ_DEV void kscale(uint32_t s0, uint32_t s1, uint32_t s2, int is, int& sc, int& m) {
  if (is < 4) {
    const int sh = 8 * is;
    sc = (s0 >> sh) & 63;
    m = (s1 >> sh) & 63;
  } else {
    const int sh = 8 * (is - 4);
    const uint32_t hi = (s2 >> sh) & 0xFF;
    sc = (hi & 0xF) | (((s0 >> sh) >> 6 & 3) << 4);
    m = (hi >> 4) | (((s1 >> sh) >> 6 & 3) << 4);
  }
}

// ---------------------------------------------------------------- Q4_0 / IQ4_NL (32-weight blocks)
template <bool NL>
struct T4Block {
  struct W { int4 q; float d; };
  struct X { int4 a, b; float d; };
  static constexpr int WT = NL ? W_IQ4_NL : W_Q4_0;
  static BARQ_DEV W load_w(const QW& w, int row, int p) {
    W r;
    const int kg = p >> 1, bi = p & 1;
    r.q = ldg16_stream(plane_chunk<WT, 0>(w, row, kg, bi));
    r.d = h2f(__ldg(reinterpret_cast<const uint16_t*>(chunk_ptr<WT>(w, row >> 7, kg) + TileFmt<WT>::D_OFF +
                                                      (row & 127) * 4) + bi));
    return r;
  }
  // Part q (0..1) of row r from a chunk staged in shared memory.
  static BARQ_DEV W load_s(const uint8_t* ch, int r, int q) {
    W s;
    s.q = *reinterpret_cast<const int4*>(staged_chunk<WT, 0>(ch, r, q));
    s.d = h2f(reinterpret_cast<const uint16_t*>(ch + TileFmt<WT>::D_OFF)[2 * r + q]);
    return s;
  }
  static BARQ_DEV X load_x(const int8_t* xq, const float2* xs, int p) {
    X x;
    x.a = ld_x16(xq + 32 * p);
    x.b = ld_x16(xq + 32 * p + 16);
    x.d = xs[p].x;
    return x;
  }
  static BARQ_DEV float dot(const W& w, const X& x, int /*lane*/) {
    int4 lo = nib_lo(w.q), hi = nib_hi(w.q);
    if (NL) {
      const int t0 = 0xBFAD9881, t1 = 0xF6EADDCF, t2 = 0x26190D01, t3 = 0x71594535;
      lo = make_int4(lut16(lo.x, t0, t1, t2, t3), lut16(lo.y, t0, t1, t2, t3), lut16(lo.z, t0, t1, t2, t3),
                     lut16(lo.w, t0, t1, t2, t3));
      hi = make_int4(lut16(hi.x, t0, t1, t2, t3), lut16(hi.y, t0, t1, t2, t3), lut16(hi.z, t0, t1, t2, t3),
                     lut16(hi.w, t0, t1, t2, t3));
    } else {
      lo = vsub4(lo, 0x08080808);
      hi = vsub4(hi, 0x08080808);
    }
    int s = dot16(lo, x.a) + dot16(hi, x.b);
    return w.d * x.d * (float)s;
  }
};

// ---------------------------------------------------------------- Q8_0
struct TQ8_0 {
  struct W { int4 a, b; float d; };
  struct X { int4 a, b; float d; };
  static BARQ_DEV W load_w(const QW& w, int row, int p) {
    W r;
    const int kg = p >> 1, bi = p & 1;
    r.a = ldg16_stream(plane_chunk<W_Q8_0, 0>(w, row, kg, 2 * bi));
    r.b = ldg16_stream(plane_chunk<W_Q8_0, 0>(w, row, kg, 2 * bi + 1));
    r.d = h2f(__ldg(reinterpret_cast<const uint16_t*>(chunk_ptr<W_Q8_0>(w, row >> 7, kg) + TileFmt<W_Q8_0>::D_OFF +
                                                      (row & 127) * 4) + bi));
    return r;
  }
  static BARQ_DEV W load_s(const uint8_t* ch, int r, int q) {
    W s;
    s.a = *reinterpret_cast<const int4*>(staged_chunk<W_Q8_0, 0>(ch, r, 2 * q));
    s.b = *reinterpret_cast<const int4*>(staged_chunk<W_Q8_0, 0>(ch, r, 2 * q + 1));
    s.d = h2f(reinterpret_cast<const uint16_t*>(ch + TileFmt<W_Q8_0>::D_OFF)[2 * r + q]);
    return s;
  }
  static BARQ_DEV X load_x(const int8_t* xq, const float2* xs, int p) {
    X x;
    x.a = ld_x16(xq + 32 * p);
    x.b = ld_x16(xq + 32 * p + 16);
    x.d = xs[p].x;
    return x;
  }
  static BARQ_DEV float dot(const W& w, const X& x, int) {
    return w.d * x.d * (float)(dot16(w.a, x.a) + dot16(w.b, x.b));
  }
};

// ---------------------------------------------------------------- Q4_K / Q5_K
// Part p of a super-block b: j = (p%8)/2 selects the 32-byte qs chunk (sub-blocks 2j and 2j+1),
// h = p%2 its 16-byte half: low nibbles are weights 64j+16h+[0,16), high nibbles 64j+32+16h+[0,16).
template <bool FIVE>
struct TK45 {
  struct W { int4 q; int4 hdr; int4 qh; };
  struct X { int4 a, b; float2 sa, sb; };
  static constexpr int WT = FIVE ? W_Q5_K : W_Q4_K;
  static BARQ_DEV W load_w(const QW& w, int row, int p) {
    W r;
    const int kg = p >> 3;
    r.q = ldg16_stream(plane_chunk<WT, 0>(w, row, kg, p & 7));
    if constexpr (FIVE) {
      r.hdr = ldg16(plane_chunk<WT, 2>(w, row, kg, 0));
      r.qh = ldg16(plane_chunk<WT, 1>(w, row, kg, p & 1));
    } else {
      r.hdr = ldg16(plane_chunk<WT, 1>(w, row, kg, 0));
    }
    return r;
  }
  static BARQ_DEV W load_s(const uint8_t* ch, int r, int q) {
    W s;
    s.q = *reinterpret_cast<const int4*>(staged_chunk<WT, 0>(ch, r, q));
    if constexpr (FIVE) {
      s.hdr = *reinterpret_cast<const int4*>(staged_chunk<WT, 2>(ch, r, 0));
      s.qh = *reinterpret_cast<const int4*>(staged_chunk<WT, 1>(ch, r, q & 1));
    } else {
      s.hdr = *reinterpret_cast<const int4*>(staged_chunk<WT, 1>(ch, r, 0));
    }
    return s;
  }
  // Parts [Q0, Q0+NQ) (NQ even: whole 32-byte qs pairs j = Q0/2 ..) of row r of a staged chunk
  // (super-block kg) against BS tokens; scales decoded once and reused for every token.
  template <int Q0, int NQ, int BS, bool X2>
  static BARQ_DEV void chunk_dot(const uint8_t* ch, int r, int kg, const ActQ8& x, int K, int nparts, int B,
                                 float* acc) {
    static_assert(Q0 % 2 == 0 && NQ % 2 == 0, "whole qs pairs");
    constexpr int J0 = Q0 / 2, NJ = NQ / 2;
    constexpr int HP = FIVE ? 2 : 1;
    const uint4 hd = *reinterpret_cast<const uint4*>(staged_chunk<WT, HP>(ch, r, 0));
    const float d = h2f(hd.x & 0xFFFF), dmin = h2f(hd.x >> 16);
    float dsc[2 * NJ], dmn[2 * NJ];
#pragma unroll
    for (int i = 0; i < 2 * NJ; ++i) {
      int sc, m;
      kscale(hd.y, hd.z, hd.w, 2 * J0 + i, sc, m);
      dsc[i] = d * (float)sc;
      dmn[i] = dmin * (float)m;
    }
    int4 qh0 = make_int4(0, 0, 0, 0), qh1 = qh0;
    if constexpr (FIVE) {
      qh0 = *reinterpret_cast<const int4*>(staged_chunk<WT, 1>(ch, r, 0));
      qh1 = *reinterpret_cast<const int4*>(staged_chunk<WT, 1>(ch, r, 1));
    }
#pragma unroll
    for (int jj = 0; jj < NJ; ++jj) {
      const int j = J0 + jj;  // qs bytes [32j, 32j+32): low nibbles sub-block 2j, high 2j+1
      const int4 q0 = *reinterpret_cast<const int4*>(staged_chunk<WT, 0>(ch, r, 2 * j));
      const int4 q1 = *reinterpret_cast<const int4*>(staged_chunk<WT, 0>(ch, r, 2 * j + 1));
      int4 a0 = nib_lo(q0), a1 = nib_lo(q1), b0 = nib_hi(q0), b1 = nib_hi(q1);
      if constexpr (FIVE) {
        const int sa = 2 * j, sb = 2 * j + 1;
        a0 = make_int4(a0.x | (((qh0.x >> sa) & 0x01010101) << 4), a0.y | (((qh0.y >> sa) & 0x01010101) << 4),
                       a0.z | (((qh0.z >> sa) & 0x01010101) << 4), a0.w | (((qh0.w >> sa) & 0x01010101) << 4));
        a1 = make_int4(a1.x | (((qh1.x >> sa) & 0x01010101) << 4), a1.y | (((qh1.y >> sa) & 0x01010101) << 4),
                       a1.z | (((qh1.z >> sa) & 0x01010101) << 4), a1.w | (((qh1.w >> sa) & 0x01010101) << 4));
        b0 = make_int4(b0.x | (((qh0.x >> sb) & 0x01010101) << 4), b0.y | (((qh0.y >> sb) & 0x01010101) << 4),
                       b0.z | (((qh0.z >> sb) & 0x01010101) << 4), b0.w | (((qh0.w >> sb) & 0x01010101) << 4));
        b1 = make_int4(b1.x | (((qh1.x >> sb) & 0x01010101) << 4), b1.y | (((qh1.y >> sb) & 0x01010101) << 4),
                       b1.z | (((qh1.z >> sb) & 0x01010101) << 4), b1.w | (((qh1.w >> sb) & 0x01010101) << 4));
      }
#pragma unroll
      for (int b = 0; b < BS; ++b) {
        if (b < B) {
          const size_t e = (size_t)b * K + 256 * kg + 64 * j;
          const int sA = dot32x<X2>(a0, a1, x.q + e, X2 ? x.ql + e : nullptr);
          const int sB = dot32x<X2>(b0, b1, x.q + e + 32, X2 ? x.ql + e + 32 : nullptr);
          const float2 xa = x.s[(size_t)b * nparts + 8 * kg + 2 * j], xb = x.s[(size_t)b * nparts + 8 * kg + 2 * j + 1];
          const float f = X2 ? (1.0f / 256.0f) : 1.0f;
          acc[b] += dsc[2 * jj] * (xa.x * f) * (float)sA + dsc[2 * jj + 1] * (xb.x * f) * (float)sB -
                    dmn[2 * jj] * xa.y - dmn[2 * jj + 1] * xb.y;
        }
      }
    }
  }
  static BARQ_DEV X load_x(const int8_t* xq, const float2* xs, int p) {
    int b = p >> 3, j = (p & 7) >> 1, h = p & 1;
    X x;
    x.a = ld_x16(xq + 256 * b + 64 * j + 16 * h);
    x.b = ld_x16(xq + 256 * b + 64 * j + 32 + 16 * h);
    x.sa = xs[8 * b + 2 * j];
    x.sb = xs[8 * b + 2 * j + 1];
    return x;
  }
  static BARQ_DEV float dot(const W& w, const X& x, int lane) {
    int j = (lane & 7) >> 1, h = lane & 1;
    int4 lo = nib_lo(w.q), hi = nib_hi(w.q);
    if (FIVE) {
      int sl = 2 * j, sh = 2 * j + 1;
      lo.x |= ((w.qh.x >> sl) & 0x01010101) << 4;
      lo.y |= ((w.qh.y >> sl) & 0x01010101) << 4;
      lo.z |= ((w.qh.z >> sl) & 0x01010101) << 4;
      lo.w |= ((w.qh.w >> sl) & 0x01010101) << 4;
      hi.x |= ((w.qh.x >> sh) & 0x01010101) << 4;
      hi.y |= ((w.qh.y >> sh) & 0x01010101) << 4;
      hi.z |= ((w.qh.z >> sh) & 0x01010101) << 4;
      hi.w |= ((w.qh.w >> sh) & 0x01010101) << 4;
    }
    int s0 = dot16(lo, x.a), s1 = dot16(hi, x.b);
    uint32_t dm = (uint32_t)w.hdr.x;
    float d = h2f(dm & 0xFFFF), dmin = h2f(dm >> 16);
    int sc0, m0, sc1, m1;
    kscale(w.hdr.y, w.hdr.z, w.hdr.w, 2 * j, sc0, m0);
    kscale(w.hdr.y, w.hdr.z, w.hdr.w, 2 * j + 1, sc1, m1);
    float r = d * ((float)sc0 * x.sa.x * (float)s0 + (float)sc1 * x.sb.x * (float)s1);
    if (h == 0) r -= dmin * ((float)m0 * x.sa.y + (float)m1 * x.sb.y);
    return r;
  }
};

// ---------------------------------------------------------------- Q6_K
// Part (n, c, h) = p%8 as n*4 + c*2 + h: ql chunk [64n + 32c + 16h, +16): low nibbles are weights
// 128n + 32c + 16h + [0,16), high nibbles the same +64; qh bytes [32n + 16h, +16) bits 2c / 4+2c.
struct TQ6_K {
  struct W { int4 ql, qh; uint32_t sc; float d; };
  struct X { int4 a, b; float da, db; };
  static BARQ_DEV W load_w(const QW& w, int row, int p) {
    W r;
    const int kg = p >> 3, q = p & 7, n = q >> 2, c = (q >> 1) & 1, h = q & 1;
    r.ql = ldg16_stream(plane_chunk<W_Q6_K, 0>(w, row, kg, q));
    r.qh = ldg16(plane_chunk<W_Q6_K, 1>(w, row, kg, 2 * n + h));
    const int8_t* sc = reinterpret_cast<const int8_t*>(plane_chunk<W_Q6_K, 2>(w, row, kg, 0));
    int lo = __ldg(sc + 8 * n + 2 * c + h), hi = __ldg(sc + 8 * n + 4 + 2 * c + h);
    r.sc = (uint32_t)(lo & 0xFFFF) | ((uint32_t)hi << 16);
    r.d = h2f(__ldg(reinterpret_cast<const uint16_t*>(chunk_ptr<W_Q6_K>(w, row >> 7, kg) + TileFmt<W_Q6_K>::D_OFF +
                                                      (row & 127) * 2)));
    return r;
  }
  static BARQ_DEV W load_s(const uint8_t* ch, int r, int q) {
    W s;
    const int n = q >> 2, c = (q >> 1) & 1, h = q & 1;
    s.ql = *reinterpret_cast<const int4*>(staged_chunk<W_Q6_K, 0>(ch, r, q));
    s.qh = *reinterpret_cast<const int4*>(staged_chunk<W_Q6_K, 1>(ch, r, 2 * n + h));
    const int8_t* sc = reinterpret_cast<const int8_t*>(staged_chunk<W_Q6_K, 2>(ch, r, 0));
    int lo = sc[8 * n + 2 * c + h], hi = sc[8 * n + 4 + 2 * c + h];
    s.sc = (uint32_t)(lo & 0xFFFF) | ((uint32_t)hi << 16);
    s.d = h2f(reinterpret_cast<const uint16_t*>(ch + TileFmt<W_Q6_K>::D_OFF)[r]);
    return s;
  }
  // Parts [Q0, Q0+NQ) of row r of a staged chunk against BS tokens; part q = 4n + 2c + h.
  template <int Q0, int NQ, int BS, bool X2>
  static BARQ_DEV void chunk_dot(const uint8_t* ch, int r, int kg, const ActQ8& x, int K, int nparts, int B,
                                 float* acc) {
    const float d = h2f(reinterpret_cast<const uint16_t*>(ch + TileFmt<W_Q6_K>::D_OFF)[r]);
    const int8_t* scp = reinterpret_cast<const int8_t*>(staged_chunk<W_Q6_K, 2>(ch, r, 0));
    const int4 sc4 = *reinterpret_cast<const int4*>(scp);  // 16 int8 scales (the plane row is one 16-byte piece)
    const int8_t* sc = reinterpret_cast<const int8_t*>(&sc4);
#pragma unroll
    for (int qi = 0; qi < NQ; ++qi) {
      {
        const int q = Q0 + qi, H = q >> 2, c = (q >> 1) & 1, h = q & 1;
        const int4 ql = *reinterpret_cast<const int4*>(staged_chunk<W_Q6_K, 0>(ch, r, q));
        const int4 qh = *reinterpret_cast<const int4*>(staged_chunk<W_Q6_K, 1>(ch, r, 2 * H + h));
        const int s_lo = 2 * c, s_hi = 4 + 2 * c;
        int4 lo = nib_lo(ql), hi = nib_hi(ql);
        lo = make_int4(lo.x | (((qh.x >> s_lo) & 0x03030303) << 4), lo.y | (((qh.y >> s_lo) & 0x03030303) << 4),
                       lo.z | (((qh.z >> s_lo) & 0x03030303) << 4), lo.w | (((qh.w >> s_lo) & 0x03030303) << 4));
        hi = make_int4(hi.x | (((qh.x >> s_hi) & 0x03030303) << 4), hi.y | (((qh.y >> s_hi) & 0x03030303) << 4),
                       hi.z | (((qh.z >> s_hi) & 0x03030303) << 4), hi.w | (((qh.w >> s_hi) & 0x03030303) << 4));
        lo = vsub4(lo, 0x20202020);
        hi = vsub4(hi, 0x20202020);
        const float dlo = d * (float)sc[8 * H + 2 * c + h], dhi = d * (float)sc[8 * H + 4 + 2 * c + h];
#pragma unroll
        for (int b = 0; b < BS; ++b) {
          if (b < B) {
            const size_t e = (size_t)b * K + 256 * kg + 128 * H + 32 * c + 16 * h;
            const int sL = dot16x<X2>(lo, x.q + e, X2 ? x.ql + e : nullptr);
            const int sH = dot16x<X2>(hi, x.q + e + 64, X2 ? x.ql + e + 64 : nullptr);
            const float f = X2 ? (1.0f / 256.0f) : 1.0f;
            const float xl = x.s[(size_t)b * nparts + 8 * kg + 4 * H + c].x * f;
            const float xh = x.s[(size_t)b * nparts + 8 * kg + 4 * H + 2 + c].x * f;
            acc[b] += dlo * xl * (float)sL + dhi * xh * (float)sH;
          }
        }
      }
    }
  }
  static BARQ_DEV X load_x(const int8_t* xq, const float2* xs, int p) {
    int b = p >> 3, q = p & 7, n = q >> 2, c = (q >> 1) & 1, h = q & 1;
    int e = 256 * b + 128 * n + 32 * c + 16 * h;
    X x;
    x.a = ld_x16(xq + e);
    x.b = ld_x16(xq + e + 64);
    x.da = xs[8 * b + 4 * n + c].x;
    x.db = xs[8 * b + 4 * n + 2 + c].x;
    return x;
  }
  static BARQ_DEV float dot(const W& w, const X& x, int lane) {
    int c = (lane >> 1) & 1;
    int s_lo = 2 * c, s_hi = 4 + 2 * c;
    int4 lo = nib_lo(w.ql), hi = nib_hi(w.ql);
    lo.x |= ((w.qh.x >> s_lo) & 0x03030303) << 4;
    lo.y |= ((w.qh.y >> s_lo) & 0x03030303) << 4;
    lo.z |= ((w.qh.z >> s_lo) & 0x03030303) << 4;
    lo.w |= ((w.qh.w >> s_lo) & 0x03030303) << 4;
    hi.x |= ((w.qh.x >> s_hi) & 0x03030303) << 4;
    hi.y |= ((w.qh.y >> s_hi) & 0x03030303) << 4;
    hi.z |= ((w.qh.z >> s_hi) & 0x03030303) << 4;
    hi.w |= ((w.qh.w >> s_hi) & 0x03030303) << 4;
    lo = vsub4(lo, 0x20202020);
    hi = vsub4(hi, 0x20202020);
    int sa = dot16(lo, x.a), sb = dot16(hi, x.b);
    float sc_lo = (float)(int16_t)(w.sc & 0xFFFF), sc_hi = (float)(int16_t)(w.sc >> 16);
    return w.d * (sc_lo * x.da * (float)sa + sc_hi * x.db * (float)sb);
  }
};

}  // namespace barq
