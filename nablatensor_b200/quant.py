"""Tape producers for the equity Monte-Carlo products (the L5 front-end).

Restates, node for node, the recording order of
  nablatensor-quant/.../quant/Products.java:70-161 (european, asian),
  nablatensor-quant/.../quant/GbmPath.java:48-91 (uniform-grid GBM step),
  nablatensor-quant/.../quant/ExoticProducts.java:55-75 (smoothed barrier),
  nablatensor-ops/.../ops/Smooth.java:44-68 (logistic step),
  nablatensor-quant/.../quant/CorrelatedNormals.java:36-93 (Cholesky mix),
  nablatensor-core/.../engine/Nabla.java:201-207 (market inputs first, in the
  market class's field order).
These run unchanged above the engine boundary in the reference; here they
produce the tapes the B200 engine replays.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, fields
from enum import Enum
from typing import Callable, List, Sequence

import numpy as np

from .tape import AadRecorder, AadTape, ADouble


@dataclass(frozen=True)
class EquityMarket:
    """EquityMarket.java: field order spot, strike, vol, rate, maturity."""
    spot: float
    strike: float
    vol: float
    rate: float
    maturity: float

    @staticmethod
    def atm_one_year() -> "EquityMarket":
        return EquityMarket(100.0, 100.0, 0.20, 0.03, 1.0)

    def validated(self) -> "EquityMarket":
        if not (self.vol >= 0.0) or not (self.maturity >= 0.0) or not (self.spot > 0.0) or not (self.strike > 0.0):
            raise ValueError(f"need spot>0, strike>0, vol>=0, maturity>=0; got {self}")
        return self


class Inputs:
    """Nabla.Inputs: one INPUT node per market field, recorded first."""

    def __init__(self, rec: AadRecorder, market):
        self._names = [f.name for f in fields(market)]
        self._nodes = [rec.input(n, float(getattr(market, n))) for n in self._names]

    def of(self, name: str) -> ADouble:
        return self._nodes[self._names.index(name)]


class TimeGrid:
    """TimeGrid.uniform(n): n equal fractions 1.0 / n."""

    def __init__(self, fractions: Sequence[float], uniform: bool):
        self.fractions = list(fractions)
        self.uniform = uniform

    @staticmethod
    def uniform_grid(n: int) -> "TimeGrid":
        if n < 1:
            raise ValueError(f"steps must be >= 1, got {n}")
        return TimeGrid([1.0 / n] * n, True)

    def steps(self) -> int:
        return len(self.fractions)


class GbmPath:
    """GbmPath (GbmPath.java:48-91)."""

    def __init__(self, rec: AadRecorder, rate: ADouble, vol: ADouble, grid: TimeGrid, maturity: ADouble):
        n = grid.steps()
        half_var = rate.sub(vol.mul(vol).mul(0.5))
        if grid.uniform:
            dt = maturity.mul(grid.fractions[0])
            d = half_var.mul(dt)
            s = vol.mul(dt.sqrt())
            self.drift = [d] * n
            self.diffusion = [s] * n
        else:
            self.drift, self.diffusion = [], []
            for i in range(n):
                dt = maturity.mul(grid.fractions[i])
                self.drift.append(half_var.mul(dt))
                self.diffusion.append(vol.mul(dt.sqrt()))

    def step(self, spot: ADouble, z: ADouble, i: int) -> ADouble:
        return spot.mul(self.drift[i].add(self.diffusion[i].mul(z)).exp())


class OptionType(Enum):
    CALL = 1
    PUT = 0


class Barrier(Enum):
    """BarrierEnum order: UP_OUT, UP_IN, DOWN_OUT, DOWN_IN."""
    UP_OUT = 0
    UP_IN = 1
    DOWN_OUT = 2
    DOWN_IN = 3


class _Sim:
    """The shared set-up of Products / ExoticProducts (their private Sim)."""

    def __init__(self, rec: AadRecorder, inp: Inputs, grid: TimeGrid):
        self.spot = inp.of("spot")
        self.strike = inp.of("strike")
        self.rate = inp.of("rate")
        self.maturity = inp.of("maturity")
        self.model = GbmPath(rec, self.rate, inp.of("vol"), grid, self.maturity)

    def discount(self, payoff: ADouble) -> ADouble:
        return payoff.mul(self.rate.neg().mul(self.maturity).exp())


def _intrinsic(kind: OptionType, underlying: ADouble, strike: ADouble) -> ADouble:
    diff = underlying.sub(strike) if kind == OptionType.CALL else strike.sub(underlying)
    return diff.max(0.0)


class Smooth:
    """Smooth.java:44-68."""

    @staticmethod
    def step(rec: AadRecorder, x: ADouble, width: float) -> ADouble:
        if not (width > 0.0) or math.isinf(width):
            raise ValueError("width must be positive and finite")
        e = x.div(width).neg().exp()
        return rec.constant(1.0).div(e.add(1.0))

    @staticmethod
    def gt(rec: AadRecorder, a: ADouble, level, width: float) -> ADouble:
        return Smooth.step(rec, a.sub(level), width)

    @staticmethod
    def lt(rec: AadRecorder, a: ADouble, level, width: float) -> ADouble:
        if isinstance(level, ADouble):
            return Smooth.step(rec, level.sub(a), width)
        return Smooth.step(rec, a.neg().add(level), width)


Product = Callable[[AadRecorder, Inputs, TimeGrid], None]


class Products:
    """Products.java: European and arithmetic-average Asian options."""

    @staticmethod
    def european(kind: OptionType = OptionType.CALL) -> Product:
        def record(rec, inp, grid):
            sim = _Sim(rec, inp, grid)
            terminal = sim.spot
            for t in range(grid.steps()):
                terminal = sim.model.step(terminal, rec.randn(), t)
            rec.output(sim.discount(_intrinsic(kind, terminal, sim.strike)))
        return record

    @staticmethod
    def asian(kind: OptionType = OptionType.CALL) -> Product:
        def record(rec, inp, grid):
            sim = _Sim(rec, inp, grid)
            path = sim.spot
            total = rec.constant(0.0)
            for t in range(grid.steps()):
                path = sim.model.step(path, rec.randn(), t)
                total = total.add(path)
            average = total.div(float(grid.steps()))
            rec.output(sim.discount(_intrinsic(kind, average, sim.strike)))
        return record

    @staticmethod
    def asian_call() -> Product:
        return Products.asian(OptionType.CALL)

    @staticmethod
    def european_call() -> Product:
        return Products.european(OptionType.CALL)


class ExoticProducts:
    """ExoticProducts.createBarrier (ExoticProducts.java:55-75)."""

    @staticmethod
    def barrier(kind: OptionType, barrier_kind: Barrier, level: float, width: float) -> Product:
        def record(rec, inp, grid):
            sim = _Sim(rec, inp, grid)
            path = sim.spot
            survival = rec.constant(1.0)
            up = barrier_kind in (Barrier.UP_OUT, Barrier.UP_IN)
            for t in range(grid.steps()):
                path = sim.model.step(path, rec.randn(), t)
                not_breached = Smooth.lt(rec, path, level, width) if up else Smooth.gt(rec, path, level, width)
                survival = survival.mul(not_breached)
            vanilla = path.sub(sim.strike).max(0.0) if kind == OptionType.CALL else sim.strike.sub(path).max(0.0)
            knock_out = barrier_kind in (Barrier.UP_OUT, Barrier.DOWN_OUT)
            alive = survival if knock_out else rec.constant(1.0).sub(survival)
            rec.output(sim.discount(vanilla.mul(alive)))
        return record


class CorrelatedNormals:
    """CorrelatedNormals.java:36-93: lower Cholesky factor of a correlation
    matrix; mix() records y = L z node by node."""

    def __init__(self, lower):
        self.lower = lower

    @staticmethod
    def of(corr) -> "CorrelatedNormals":
        n = len(corr)
        lo = [[0.0] * n for _ in range(n)]
        for i in range(n):
            for j in range(i + 1):
                s = float(corr[i][j])
                for k in range(j):
                    s -= lo[i][k] * lo[j][k]
                if i == j:
                    if s <= 0.0:
                        raise ValueError(f"correlation matrix is not positive definite at index {i}")
                    lo[i][j] = math.sqrt(s)
                else:
                    lo[i][j] = s / lo[j][j]
        return CorrelatedNormals(lo)

    def size(self) -> int:
        return len(self.lower)

    def mix(self, rec: AadRecorder, z: Sequence[ADouble]) -> List[ADouble]:
        y = []
        for i in range(len(self.lower)):
            acc = rec.constant(0.0)
            for j in range(i + 1):
                acc = acc.add(z[j].mul(self.lower[i][j]))
            y.append(acc)
        return y

    def draw(self, rec: AadRecorder) -> List[ADouble]:
        return self.mix(rec, [rec.randn() for _ in range(len(self.lower))])


def equicorrelation(n: int, rho: float):
    return [[1.0 if i == j else rho for j in range(n)] for i in range(n)]


class BasketOption:
    """An n-asset arithmetic basket option under correlated GBM.  The reference
    fixes the basket at 3 assets (BasketOption.java:35-76); this records the
    same per-step shape for any n: market inputs s_1..s_n, v_1..v_n, rate (in
    that order), a Cholesky mix of n fresh normals per step, then per asset
    s_i *= exp(drift_i + v_i sqrt(dt) y_i)."""

    @staticmethod
    def record(rec: AadRecorder, spots, vols, rate: float, weights, strike: float, corr, maturity: float,
               steps: int, kind: OptionType = OptionType.CALL) -> None:
        n = len(spots)
        mixer = CorrelatedNormals.of(corr)
        dt = maturity / steps
        sqrt_dt = math.sqrt(dt)
        s = [rec.input(f"s{i + 1}", float(spots[i])) for i in range(n)]
        vol = [rec.input(f"v{i + 1}", float(vols[i])) for i in range(n)]
        r = rec.input("rate", float(rate))
        drift = [r.sub(vol[i].mul(vol[i]).mul(0.5)).mul(dt) for i in range(n)]
        for _ in range(steps):
            z = mixer.draw(rec)
            for i in range(n):
                s[i] = s[i].mul(drift[i].add(vol[i].mul(sqrt_dt).mul(z[i])).exp())
        level = rec.constant(0.0)
        for i in range(n):
            level = level.add(s[i].mul(float(weights[i])))
        intrinsic = level.sub(strike).max(0.0) if kind == OptionType.CALL else rec.constant(strike).sub(level).max(0.0)
        rec.output(intrinsic.mul(r.neg().mul(maturity).exp()))


def basket_config4_market(n: int = 10, seed: int = 7):
    """Benchmark configuration 4's market: spots ~ U[80, 120] and vols ~ U[0.15, 0.40],
    drawn with numpy's PCG64 generator seeded 7 (spots first, then vols)."""
    g = np.random.Generator(np.random.PCG64(seed))
    spots = g.uniform(80.0, 120.0, n)
    vols = g.uniform(0.15, 0.40, n)
    return [float(x) for x in spots], [float(x) for x in vols]


def basket_tape(n: int = 10, steps: int = 52, rho: float = 0.5, seed: int = 7, strike: float = 100.0,
                rate: float = 0.03, maturity: float = 1.0) -> AadTape:
    """Benchmark configuration 4: 10-asset equal-weight basket call, equicorrelation
    0.5, 52 weekly steps, T = 1; 21 Greeks (10 spots, 10 vols, rate)."""
    spots, vols = basket_config4_market(n, seed)
    return AadRecorder.record(lambda rec: BasketOption.record(
        rec, spots, vols, rate, [1.0 / n] * n, strike, equicorrelation(n, rho), maturity, steps))


def record_model(market, product: Product, grid: TimeGrid) -> AadTape:
    """Nabla.model(market, (rec, in) -> product.record(rec, in, grid)).tape()."""
    def body(rec):
        product(rec, Inputs(rec, market), grid)
    return AadRecorder.record(body)


def asian_tape(steps: int = 252, market: EquityMarket = None) -> AadTape:
    return record_model(market or EquityMarket.atm_one_year(), Products.asian_call(), TimeGrid.uniform_grid(steps))


def european_tape(steps: int = 1, market: EquityMarket = None) -> AadTape:
    return record_model(market or EquityMarket.atm_one_year(), Products.european_call(), TimeGrid.uniform_grid(steps))


def barrier_tape(steps: int = 252, level: float = 80.0, width: float = 1.0, kind: Barrier = Barrier.DOWN_IN,
                 option: OptionType = OptionType.CALL, market: EquityMarket = None) -> AadTape:
    return record_model(market or EquityMarket.atm_one_year(), ExoticProducts.barrier(option, kind, level, width),
                        TimeGrid.uniform_grid(steps))


# ---- CVA of an interest-rate swap book under one-factor Hull-White --------------
#
# The reference records CVA path by path and trade by trade
# (nablatensor-cva/.../ExposureSimulation.java:121-229, InterestRateSwap.java:129-154,
# HwShortRate.java): every exposure date values each swap's remaining coupons, so
# no two dates record the same nodes.  The book here is the benchmark configuration 5
# book -- 100 spot-starting payer swaps on a semi-annual grid, a 40-pillar zero
# curve -- and its netted value is the same sum regrouped by payment date, so
# every monthly date records one identical body and only its constants change
# (which coupons are still alive, the bond coefficients of that date).  The
# loop planner then keeps those constants in a per-date table.
#
#   x_k   = x_{k-1} e^{-a dt} + sigma sqrt((1 - e^{-2a dt}) / 2a) z_k   (exact OU step)
#   I_k   = I_{k-1} + (x_{k-1} + x_k) dt / 2                           (integral of x)
#   lp_k  = ln P(0, t_k), from the two pillar zero rates around t_k    (before the loop, gathered per date)
#   P_kj  = P(t_k, T_j) = exp(lp(T_j) - lp_k + A(t_k, T_j) - B(t_k, T_j) x_k)
#   V_k   = A0_k - sum_j W_kj P_kj                                     (netted payer value, in millions)
#   D_k   = exp(lp_k - I_k - V(0, t_k) / 2)                              (stochastic discount)
#   CVA  += LGD max(V_k, 0) D_k S_{k-1} (1 - e^{-lambda dt}),   S_k = S_{k-1} e^{-lambda dt}
#
# with B, A and V(t, T) the Hull-White x-representation coefficients
# (Brigo and Mercurio, Interest Rate Models, 2nd ed., section 3.3).

MONEY_UNIT = 1.0e6  # the tape carries values in millions (ExposureSimulation.java:61-69)


@dataclass
class SwapBook:
    notional: np.ndarray   # per swap
    fixed_rate: np.ndarray
    maturity: np.ndarray   # years, on the semi-annual payment grid

    @staticmethod
    def config5(n: int = 100, seed: int = 11, accrual: float = 0.5) -> "SwapBook":
        g = np.random.Generator(np.random.PCG64(seed + 1))
        notional = g.uniform(1e6, 1e8, n)
        fixed = g.normal(0.03, 0.005, n)
        mat = np.clip(np.round(g.uniform(1.0, 10.0, n) / accrual) * accrual, accrual, 10.0)
        return SwapBook(notional, fixed, mat)


def cva_config5_curve(pillars: int = 40, seed: int = 11):
    """Zero rates at T_i = 0.25 i: flat 3% + N(0, 25bp), PCG64 seed 11."""
    g = np.random.Generator(np.random.PCG64(seed))
    return [0.25 * (i + 1) for i in range(pillars)], [float(z) for z in 0.03 + g.normal(0.0, 0.0025, pillars)]


def _curve_weights(t: float, tenors: Sequence[float]) -> np.ndarray:
    """ln P(0, t) = -t zeta(t) as weights on the pillar zero rates: zeta
    linear between pillars, flat outside."""
    w = np.zeros(len(tenors))
    if t <= tenors[0]:
        w[0] = -t
    elif t >= tenors[-1]:
        w[-1] = -t
    else:
        i = int(np.searchsorted(tenors, t)) - 1
        f = (t - tenors[i]) / (tenors[i + 1] - tenors[i])
        w[i], w[i + 1] = -t * (1.0 - f), -t * f
    return w


def cva_tape(dates: int = 120, horizon: float = 10.0, a: float = 0.05, sigma: float = 0.01, hazard: float = 0.02,
             recovery: float = 0.4, book: SwapBook = None, pillars: int = 40, seed: int = 11,
             accrual: float = 0.5) -> AadTape:
    """Benchmark configuration 5: CVA of the swap book, adjoints w.r.t. the pillar zero
    rates and the hazard rate (41 inputs)."""
    book = book if book is not None else SwapBook.config5(seed=seed, accrual=accrual)
    tenors, zeros = cva_config5_curve(pillars, seed)
    dt = horizon / dates
    pay = [accrual * (j + 1) for j in range(int(round(horizon / accrual)))]

    def Bf(t, T):
        return (1.0 - math.exp(-a * (T - t))) / a

    def Vf(t, T):
        tau = T - t
        return sigma ** 2 / a ** 2 * (tau + 2.0 / a * math.exp(-a * tau) - 0.5 / a * math.exp(-2.0 * a * tau)
                                      - 1.5 / a)

    def Af(t, T):
        return 0.5 * (Vf(t, T) - Vf(0.0, T) + Vf(0.0, t))

    ea = math.exp(-a * dt)
    sd = sigma * math.sqrt((1.0 - math.exp(-2.0 * a * dt)) / (2.0 * a))
    N = book.notional / MONEY_UNIT

    def body(rec: AadRecorder):
        zeta = [rec.input(f"zero_{T:g}y", z) for T, z in zip(tenors, zeros)]
        lam = rec.input("hazard", hazard)
        lp_pay = []
        for T in pay:
            w = _curve_weights(T, tenors)
            acc = None
            for i in np.nonzero(w)[0]:
                term = zeta[i].mul(float(w[i]))
                acc = term if acc is None else acc.add(term)
            lp_pay.append(acc)
        # ln P(0, t_k) of every exposure date, before the loop: each date's
        # body reads its own (the loop gathers them per unit).
        lp_dates = []
        for k in range(1, dates + 1):
            w = _curve_weights(k * dt, tenors)
            acc = None
            for i in np.nonzero(w)[0]:
                term = zeta[i].mul(float(w[i]))
                acc = term if acc is None else acc.add(term)
            lp_dates.append(acc)
        surv_step = lam.mul(-dt).exp()                   # e^{-lambda dt}
        pd_step = surv_step.neg().add(1.0)               # 1 - e^{-lambda dt}
        x = rec.constant(0.0)
        integ = rec.constant(0.0)
        surv = rec.constant(1.0)
        cva = rec.constant(0.0)
        for k in range(1, dates + 1):
            t = k * dt
            x_new = x.mul(ea).add(rec.randn().mul(sd))
            integ = integ.add(x.add(x_new).mul(0.5 * dt))
            x = x_new
            lp = lp_dates[k - 1]
            alive = book.maturity > t + 1e-9
            a0 = float(N[alive].sum())
            value = rec.constant(a0)
            for j, T in enumerate(pay):
                live = T > t + 1e-9
                w = 0.0
                if live:
                    coupon = alive & (book.maturity >= T - 1e-9)
                    w = float((N[coupon] * book.fixed_rate[coupon]).sum() * accrual
                              + N[alive & (np.abs(book.maturity - T) < 1e-9)].sum())
                A = Af(t, T) if live else 0.0
                Bn = -Bf(t, T) if live else 0.0
                bond = lp_pay[j].sub(lp).add(x.mul(Bn).add(A)).exp()
                value = value.sub(bond.mul(w))
            exposure = value.max(0.0)
            discount = lp.sub(integ).sub(0.5 * Vf(0.0, t)).exp()
            cva = cva.add(exposure.mul(discount).mul(surv.mul(pd_step)).mul(1.0 - recovery))
            surv = surv.mul(surv_step)
        rec.output(cva)

    return AadRecorder.record(body)


# ---- generic tapes used by the conformance tests ---------------------------------

def every_op(rec: AadRecorder) -> None:
    """A tape touching all 15 ops (the shape of AadOpConformanceTest.everyOp)."""
    x = rec.input("x", 1.3)
    y = rec.input("y", 0.7)
    z = rec.randn()
    u = rec.randu()
    a = x.add(y).sub(0.1)
    b = x.mul(y).div(x.add(0.5))
    c = a.neg().exp().add(b.abs())
    d = c.add(1.0).log().sqrt()
    e = d.max(z.mul(0.01)).min(x.mul(2.0))
    rec.output(e.add(u.mul(y)))


__all__ = ["EquityMarket", "TimeGrid", "GbmPath", "OptionType", "Barrier", "Smooth", "Products", "ExoticProducts",
           "Inputs", "record_model", "asian_tape", "european_tape", "barrier_tape", "every_op", "SwapBook",
           "cva_config5_curve", "cva_tape"]
