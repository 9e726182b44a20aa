"""A second restatement of fdlibm's exp (e_exp.c, Sun Microsystems 1993), the
method V8's Math.exp ports (V8 src/base/ieee754.cc, ieee754::exp), written in
plain Python so that it shares no code with the oracle's C restatement
(oracle/ms_oracle.c, js_exp).  Python floats are IEEE doubles and every
operator below rounds once, so this reproduces the published method bit for
bit.  Test infrastructure only.

Method: x = k*ln2 + r with |r| <= ln2/2 (ln2 = ln2_hi + ln2_lo, ln2_hi with
trailing zero bits so that k*ln2_hi is exact); on that range
r*(e^r + 1)/(e^r - 1) is approximated by 2 + P1 z + ... + P5 z^5 (z = r^2), which
gives e^r = 1 + r + r*c/(2 - c) with c = r - z*(P1 + ... ); then e^x = 2^k e^r.
"""
import math
import struct

LN2_HI = 6.93147180369123816490e-01   # high word 0x3fe62e42, low word 0xfee00000
LN2_LO = 1.90821492927058770002e-10   # 0x3dea39ef 35793c76
INV_LN2 = 1.44269504088896338700e+00  # 0x3ff71547 652b82fe
P = (1.66666666666666019037e-01, -2.77777777770155933842e-03, 6.61375632143793436117e-05,
     -1.65339022054652515390e-06, 4.13813679705723846039e-08)
OVERFLOW_AT = 7.09782712893383973096e+02
UNDERFLOW_AT = -7.45133219101941108420e+02


def _high_word(x: float) -> int:
    return struct.unpack("<Q", struct.pack("<d", x))[0] >> 32


def _low_word(x: float) -> int:
    return struct.unpack("<Q", struct.pack("<d", x))[0] & 0xFFFFFFFF


def fdlibm_exp(x: float) -> float:
    hw = _high_word(x)
    negative = hw >> 31
    ahw = hw & 0x7FFFFFFF
    if ahw >= 0x40862E42:
        if ahw >= 0x7FF00000:
            if (ahw & 0xFFFFF) | _low_word(x):
                return x + x                      # NaN
            return 0.0 if negative else x         # -inf -> 0, inf -> inf
        if x > OVERFLOW_AT:
            return math.inf
        if x < UNDERFLOW_AT:
            return 0.0
    k = 0
    hi = lo = 0.0
    if ahw > 0x3FD62E42:                          # |x| > ln2/2
        if ahw < 0x3FF0A2B2:                      # |x| < 1.5*ln2
            if x == 1.0:
                return 2.718281828459045          # V8 returns E here
            if negative:
                hi, lo, k = x + LN2_HI, -LN2_LO, -1
            else:
                hi, lo, k = x - LN2_HI, LN2_LO, 1
        else:
            k = int(INV_LN2 * x + (-0.5 if negative else 0.5))  # truncates toward zero, like C
            t = float(k)
            hi = x - t * LN2_HI
            lo = t * LN2_LO
        r = hi - lo
    elif ahw < 0x3E300000:                        # |x| < 2^-28
        return 1.0 + x
    else:
        r = x
    z = r * r
    c = r - z * (P[0] + z * (P[1] + z * (P[2] + z * (P[3] + z * P[4]))))
    if k == 0:
        return 1.0 - ((r * c) / (c - 2.0) - r)
    y = 1.0 - ((lo - (r * c) / (2.0 - c)) - hi)
    if k >= -1021:
        if k == 1024:
            return y * 2.0 * math.ldexp(1.0, 1023)
        return math.ldexp(y, k)                   # exact: the result is normal
    return math.ldexp(y, k + 1000) * math.ldexp(1.0, -1000)
