"""Test tapes beyond the equity products, each the shape of a reference test.

random_branching  CudaCheckpointParityTest.randomBranchingTapeMatchesPlain
                  (nablatensor-examples/.../CudaCheckpointParityTest.java:76-88)
every_op          AadOpConformanceTest.everyOp (AadOpConformanceTest.java:50-60)
named_streams     RandomStreamsTest.cpuAndJitAgree... (RandomStreamsTest.java:66-80)
lookback          Products.lookback (Products.java:102-117)
multi_output      two recorded outputs (AadRecorder.java:108-122)
fp32_asian_50     Fp32BackendComparisonTest.asianCall (Fp32BackendComparisonTest.java:45-59)
nonuniform_asian  an Asian call on a non-uniform TimeGrid (TimeGrid.of, TimeGrid.java): every step
                  records its own dt and sqrt(dt) constants, so the loop's constants differ per unit
term_vol_asian    an Asian call with a volatility input per step: every step reads its own input and
                  its own drift node from before the loop (gathered per unit)
"""
import math

from nablatensor_b200.quant import Smooth, every_op
from nablatensor_b200.tape import AadRecorder


def random_branching(steps=24):
    def body(rec):
        level = rec.input("level", 1.2)
        scale = rec.input("scale", 0.1)
        for _ in range(steps):
            level = level.add(rec.randn().mul(scale)).add(rec.randn().mul(0.01)).max(0.01)
        rec.output(level.log().exp().sqrt().div(scale.add(1.0)))
    return AadRecorder.record(body)


def every_op_tape():
    return AadRecorder.record(every_op)


def named_streams(steps=16):
    def body(rec):
        s0 = rec.input("S0", 100.0)
        vol = rec.input("sigma", 0.2)
        jumps = rec.stream("jump-clock")
        acc = s0
        for _ in range(steps):
            z = rec.randn()
            u = jumps.randu()
            jump = Smooth.gt(rec, u, 0.97, 0.01)
            acc = acc.mul(vol.mul(z).mul(0.05).add(1.0)).add(jump.mul(2.0))
        rec.output(acc)
    return AadRecorder.record(body)


def lookback(steps=64, call=True):
    def body(rec):
        spot = rec.input("spot", 100.0)
        strike = rec.input("strike", 100.0)
        vol = rec.input("vol", 0.20)
        rate = rec.input("rate", 0.03)
        mat = rec.input("maturity", 1.0)
        half_var = rate.sub(vol.mul(vol).mul(0.5))
        dt = mat.mul(1.0 / steps)
        drift = half_var.mul(dt)
        diff = vol.mul(dt.sqrt())
        path = spot
        ext = spot
        for _ in range(steps):
            path = path.mul(drift.add(diff.mul(rec.randn())).exp())
            ext = ext.max(path) if call else ext.min(path)
        intrinsic = ext.sub(strike).max(0.0) if call else strike.sub(ext).max(0.0)
        rec.output(intrinsic.mul(rate.neg().mul(mat).exp()))
    return AadRecorder.record(body)


def multi_output(steps=40):
    def body(rec):
        spot = rec.input("spot", 100.0)
        vol = rec.input("vol", 0.25)
        path = spot
        total = rec.constant(0.0)
        for _ in range(steps):
            path = path.mul(vol.mul(rec.randn()).mul(0.1).add(1.0))
            total = total.add(path)
        rec.output("terminal", path.sub(95.0).max(0.0))
        rec.output("average", total.div(float(steps)).sub(100.0).abs())
    return AadRecorder.record(body)


def fp32_asian_50(fixings=50):
    S0, K, VOL, RATE, T = 100.0, 100.0, 0.20, 0.03, 1.0

    def body(rec):
        spot = rec.input("spot", S0)
        vol = rec.input("vol", VOL)
        dt = T / fixings
        drift = vol.mul(vol).mul(-0.5 * dt).add(RATE * dt)
        diffusion = vol.mul(math.sqrt(dt))
        price = spot
        total = rec.constant(0.0)
        for _ in range(fixings):
            price = price.mul(drift.add(diffusion.mul(rec.randn())).exp())
            total = total.add(price)
        average = total.mul(1.0 / fixings)
        rec.output(average.sub(K).max(0.0).mul(math.exp(-RATE * T)))
    return AadRecorder.record(body)


def odd_steps_asian(steps=31):
    from nablatensor_b200.quant import asian_tape
    return asian_tape(steps)


def nonuniform_asian(steps=60):
    """Asian call on a grid whose step lengths grow geometrically: the step
    body is the same every step except for its dt constants."""
    w = [1.02 ** k for k in range(steps)]
    dts = [x / sum(w) for x in w]

    def body(rec):
        spot = rec.input("spot", 100.0)
        strike = rec.input("strike", 100.0)
        vol = rec.input("vol", 0.2)
        rate = rec.input("rate", 0.03)
        drift = rate.sub(vol.mul(vol).mul(0.5))
        s, acc = spot, rec.constant(0.0)
        for dt in dts:
            s = s.mul(drift.mul(dt).add(vol.mul(math.sqrt(dt)).mul(rec.randn())).exp())
            acc = acc.add(s)
        payoff = acc.div(float(steps)).sub(strike).max(0.0)
        rec.output(payoff.mul(rate.neg().exp()))
    return AadRecorder.record(body)


def term_vol_asian(steps=24):
    """Asian call with a term structure of volatility: step k reads input
    vol_k and a drift computed for it before the loop."""
    dt = 1.0 / steps

    def body(rec):
        spot = rec.input("spot", 100.0)
        strike = rec.input("strike", 100.0)
        rate = rec.input("rate", 0.03)
        vols = [rec.input(f"vol_{k}", 0.15 + 0.2 * k / steps) for k in range(steps)]
        drifts = [rate.sub(v.mul(v).mul(0.5)).mul(dt) for v in vols]
        s, acc = spot, rec.constant(0.0)
        for k in range(steps):
            s = s.mul(drifts[k].add(vols[k].mul(math.sqrt(dt)).mul(rec.randn())).exp())
            acc = acc.add(s)
        payoff = acc.div(float(steps)).sub(strike).max(0.0)
        rec.output(payoff.mul(rate.neg().exp()))
    return AadRecorder.record(body)


def pow2_divisions(steps=24, tiny=2.0 ** -1000):
    """Divisions by constants: powers of two (rewritten to a multiplication by
    the exact reciprocal: 2, 0.5, 1, -4 and `tiny`), a power of two that also
    feeds an addition (kept a division), and 3 (kept)."""
    def body(rec):
        s = rec.input("s", 1.5)
        v = rec.input("v", 0.3)
        shared = rec.constant(2.0)
        acc = s
        for _ in range(steps):
            z = rec.randn()
            x = acc.div(2.0).add(v.mul(z).div(0.5)).div(1.0).add(z.div(-4.0)).add(acc.div(3.0))
            acc = x.div(shared).add(shared).mul(0.25).add(v.div(tiny).mul(tiny))
        rec.output(acc)
    return AadRecorder.record(body)


def near_overflow_exps(steps=8, s0=699.0):
    """A loop whose taped exps (carry-dependent arguments) lie near the top of
    the double range: exp(s) for s a random walk from s0, scaled by 1e-300 so
    that the sums stay finite.  From s0 = 699 many lanes pass |x| = 700, where
    the forward loop's first-pass exp records the argument and the warp redoes
    the loop with the full-range routine; from 690 none does."""
    def body(rec):
        level = rec.input("s0", s0)
        vol = rec.input("vol", 0.3)
        acc = rec.constant(0.0)
        for _ in range(steps):
            level = level.add(rec.randn().mul(vol))
            acc = acc.add(level.exp().mul(1e-300))
        rec.output(acc)
    return AadRecorder.record(body)
