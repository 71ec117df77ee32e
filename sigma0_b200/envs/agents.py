"""Action builders and reward functions of the market-making and execution agents.

The reference's market-making environment chooses its action mapping and reward from a
config string (``src/environment/jaxen/mm_env.py:160-178`` action spaces, ``:2178-2440``
rewards and inventory penalties); its execution environment likewise
(``src/environment/jaxen/exec_env.py:160-173`` action spaces, ``:1511-1700`` the VWAP
reward).  Each builder here maps a batch of actions and the books' touch to the orders an
agent wants resting after this step, as one tensor ``(n, K, 3)`` of ``(side, price, qty)``
rows (side +1 bid / -1 ask, 0 = no order), plus optional marketable orders; the
environment cancels the agent's previous orders and submits these.  Prices are in the
engine's integer price units, quantities in shares.

Market-making action spaces (``MM_ACTION_SPACES``):

``fixed_quants``        action in [0, 8): a pair of size multiples (bid, ask) at the touch
``fixed_prices``        action (n, 2L): sizes (in quote-size units) at L bid and L ask levels
``AvSt``                action in [0, 8): the Avellaneda-Stoikov risk aversion gamma; quotes at
                        the reservation price r = mid - q gamma sigma^2 tau, +/- the optimal half
                        spread (gamma sigma^2 tau + (2 / gamma) ln(1 + gamma / k)) / 2
``bobStrategy``         action in [0, 5): inventory skew kappa; both quotes shifted against the
                        inventory by kappa * inventory / quote size ticks
``bobRL``               action (n, 2): (kappa index, size multiple index)
``spread_skew``         action (n, 2): (half spread index, skew index) around the mid
``directional_trading`` action in [0, 5): nothing, market buy, market sell, bid only, ask only
``simple``              action in [0, 4): both sides at the touch, bid only, ask only, none
``offsets``             action (n, 2): offsets (ticks) of the bid and the ask from the mid

Rewards (``MM_REWARDS``), per step and agent, in ticks:

``portfolio_value``        cash + inventory valued at the reference price
``delta_portfolio_value``  its change over the step
``buy_sell_pnl``           sum over the step's buys of (ref_buy - price) q plus over its sells
                           of (price - ref_sell) q
``spooner``                buy_sell_pnl + rebate + inventory PnL (inventory before the step
                           times the mid's move)
``spooner_damped``         spooner - eta * inventory PnL
``spooner_asym_damped``    spooner - max(0, eta * inventory PnL)
``spooner_asym_damped2``   buy_sell_pnl + rebate + gamma (inventory PnL - max(0, eta * inventory PnL))
``spooner_scaled``         buy_sell_pnl + rebate + eta (inventory PnL - (1 - eta) max(0, inventory PnL))
``complex``                spooner_asym_damped - lambda |inventory change|
``zero_inv``               -|inventory|
``pnl_inventory``          change of mark-to-market PnL at the mid (the default)
and an inventory penalty (``none`` / ``linear`` / ``quadratic`` / ``threshold`` / ``exp4``) on
top of any of them.  The reference price of the PnL terms is the mid after the step, the
step's average mid (``mid_avg``), the far or the near touch.

Execution action spaces (``EXEC_ACTION_SPACES``): ``sizes`` (a marketable child order of
a size from a table), ``fixed_quants`` (a pair (aggressive, passive) of size multiples:
marketable at the far touch, resting at the near touch), ``fixed_quants_1msg`` (one order,
action picks size and aggressiveness), ``fixed_prices`` (sizes at the far touch, the mid,
the near touch and one tick behind it), ``fixed_quants_complex`` (the reference's 13-action
ladder: nothing, or 1, 2 or 5 clips at one of those four prices), ``simplest_case`` (wait or
take one clip at the far touch) and ``twap`` (the action is ignored: target / steps at the far touch every step).
Execution rewards: ``slippage`` (negative shortfall against the arrival mid per share of
the target), the reference's ``normal``, ``finish_fast`` and ``simplest_case`` (see
``exec_reward``) and ``vwap`` (the reference's advantage over the market's VWAP of the step
plus lambda times the drift of that VWAP from the arrival price).
"""
from __future__ import annotations

from typing import Dict, Tuple

import torch

MM_ACTION_SPACES = ("offsets", "fixed_quants", "fixed_prices", "AvSt", "bobStrategy", "bobRL", "spread_skew",
                    "directional_trading", "simple")
MM_REWARDS = ("pnl_inventory", "portfolio_value", "delta_portfolio_value", "buy_sell_pnl", "spooner",
              "spooner_damped", "spooner_asym_damped", "spooner_asym_damped2", "spooner_scaled", "complex",
              "zero_inv")
EXEC_ACTION_SPACES = ("sizes", "fixed_quants", "fixed_quants_1msg", "fixed_prices", "fixed_quants_complex",
                      "simplest_case", "twap")
EXEC_REWARDS = ("slippage", "vwap", "normal", "finish_fast", "simplest_case")

OFFSETS = (1, 2, 3, 5, 8)
FIXED_QUANTS = ((1, 1), (2, 1), (1, 2), (2, 2), (1, 0), (0, 1), (2, 0), (0, 2))
AVST_GAMMAS = (0.1, 0.2, 0.5, 1.0, 2.0, 5.0, 10.0, 20.0)
KAPPAS = (0.0, 0.05, 0.1, 0.5, 0.9)
SIZE_MULTS = (1, 2, 3)
HALF_SPREADS = (1, 2, 3, 5, 8)
SKEWS = (-2, -1, 0, 1, 2)


def _rows(*orders) -> torch.Tensor:
    """Stack (side, price, qty) triples of (n,) tensors into (n, K, 3)."""
    return torch.stack([torch.stack([s, p, q], -1) for s, p, q in orders], 1).long()


def _passive(bid, ask, best_bid, best_ask, tick):
    """Keep quotes from crossing the touch (a bid above the best ask would trade)."""
    bid = torch.minimum(bid, best_ask - tick)
    ask = torch.maximum(ask, best_bid + tick)
    return bid, ask


def mm_orders(space: str, action: torch.Tensor, st: Dict[str, torch.Tensor], size: int, tick: int,
              n_levels: int = 3, avst_k: float = 1.5, avst_var: float = 2.0) -> Tuple[torch.Tensor, torch.Tensor]:
    """(orders (n, K, 3), market (n, 2) = (side, qty)) for one market maker.  ``st`` holds
    the books' best_bid, best_ask, mid (engine price units), inventory (shares) and
    time_left (fraction of the episode, in [0, 1])."""
    bb, ba, mid, inv = st["best_bid"], st["best_ask"], st["mid"], st["inventory"]
    n = mid.shape[0]
    one, zero = torch.ones_like(mid), torch.zeros_like(mid)
    market = torch.zeros(n, 2, dtype=torch.long)
    a = action.long()
    if space == "offsets":
        off = torch.tensor(OFFSETS)
        bid, ask = mid - off[a[:, 0]] * tick, mid + off[a[:, 1]] * tick
        orders = _rows((one, bid, one * size), (-one, ask, one * size))
    elif space == "fixed_quants":
        t = torch.tensor(FIXED_QUANTS)[a]
        orders = _rows((one, bb, t[:, 0] * size), (-one, ba, t[:, 1] * size))
    elif space == "fixed_prices":
        L = n_levels
        rows = [(one, bb - i * tick, a[:, i] * size) for i in range(L)]
        rows += [(-one, ba + i * tick, a[:, L + i] * size) for i in range(L)]
        orders = _rows(*rows)
    elif space == "AvSt":
        g = torch.tensor(AVST_GAMMAS, dtype=torch.float64)[a]
        tau = st["time_left"].double()
        q = inv.double() / size
        r = mid.double() / tick - q * g * avst_var * tau
        half = (g * avst_var * tau + (2.0 / g) * torch.log1p(g / avst_k)) / 2.0
        bid = torch.floor(r - half).long() * tick
        ask = torch.ceil(r + half).long() * tick
        bid, ask = _passive(bid, ask, bb, ba, tick)
        orders = _rows((one, bid, one * size), (-one, ask, one * size))
    elif space in ("bobStrategy", "bobRL"):
        ki = a if space == "bobStrategy" else a[:, 0]
        mult = one if space == "bobStrategy" else torch.tensor(SIZE_MULTS)[a[:, 1]]
        shift = torch.round(torch.tensor(KAPPAS, dtype=torch.float64)[ki] * inv.double() / size).long() * tick
        bid, ask = _passive(bb - shift, ba - shift, bb, ba, tick)
        orders = _rows((one, bid, mult * size), (-one, ask, mult * size))
    elif space == "spread_skew":
        s = torch.tensor(HALF_SPREADS)[a[:, 0]] * tick
        k = torch.tensor(SKEWS)[a[:, 1]] * tick
        bid, ask = _passive(mid - s + k, mid + s + k, bb, ba, tick)
        orders = _rows((one, bid, one * size), (-one, ask, one * size))
    elif space == "directional_trading":
        bid_q = torch.where(a == 3, one * size, zero)
        ask_q = torch.where(a == 4, one * size, zero)
        orders = _rows((one, bb, bid_q), (-one, ba, ask_q))
        market[:, 0] = torch.where(a == 1, 1, torch.where(a == 2, -1, 0))
        market[:, 1] = torch.where((a == 1) | (a == 2), size, 0)
    elif space == "simple":
        bid_q = torch.where((a == 0) | (a == 1), one * size, zero)
        ask_q = torch.where((a == 0) | (a == 2), one * size, zero)
        orders = _rows((one, bb, bid_q), (-one, ba, ask_q))
    else:
        raise ValueError(f"unknown market-making action space {space!r}; one of {MM_ACTION_SPACES}")
    # no order without a price or a size, nor on a book without a two-sided touch
    bad = (orders[..., 2] <= 0) | (orders[..., 1] <= 0) | (mid <= 0)[:, None]
    orders[bad] = 0
    market[mid <= 0] = 0
    return orders, market


def agent_trades(trades: torch.Tensor, tid: int):
    """The step's buys and sells of trader ``tid``: (buy_qty, buy_value, sell_qty, sell_value)
    per env (value = sum of price x qty).  Trade rows: price, qty, ..., passive trader id
    (column 6), aggressive trader id (column 7); the quantity is signed from the resting
    order's side, so the passive trader's signed fill (+ bought) is +qty and the aggressor's
    -qty."""
    price, q = trades[..., 0].long(), trades[..., 1].long()
    valid = price >= 0
    aggr = valid & (trades[..., 7] == tid)
    pas = valid & (trades[..., 6] == tid)
    # signed shares bought by tid: + when tid bought
    signed = torch.where(aggr, -q, torch.zeros_like(q)) + torch.where(pas, q, torch.zeros_like(q))
    bq = signed.clamp(min=0)
    sq = (-signed).clamp(min=0)
    return bq.sum(-1), (bq * price).sum(-1), sq.sum(-1), (sq * price).sum(-1)


def mm_reward(name: str, *, buy_q, buy_v, sell_q, sell_v, inv_prev, inv, cash, mid0, mid1, best_bid, best_ask,
              tick: int, reference_price: str = "mid", eta: float = 0.5, gamma: float = 1.0, lam: float = 0.0,
              rebate_bps: float = 0.0, pv_prev=None):
    """One market maker's reward for the step (ticks); see the module docstring."""
    d = torch.float64
    buy_q, sell_q, inv_prev, inv = buy_q.to(d), sell_q.to(d), inv_prev.to(d), inv.to(d)
    buy_v, sell_v, cash = buy_v.to(d), sell_v.to(d), cash.to(d)
    mid0, mid1 = mid0.to(d), mid1.to(d)
    if reference_price == "mid":
        ref_buy = ref_sell = ref = mid1
    elif reference_price == "mid_avg":       # the step's average mid (before / after the step)
        ref_buy = ref_sell = ref = (mid0 + mid1) / 2
    elif reference_price == "far_touch":
        ref_buy, ref_sell = best_ask.to(d), best_bid.to(d)
        ref = torch.where(inv > 0, best_bid.to(d), best_ask.to(d))
    elif reference_price == "near_touch":
        ref_buy, ref_sell = best_bid.to(d), best_ask.to(d)
        ref = torch.where(inv > 0, best_ask.to(d), best_bid.to(d))
    else:
        raise ValueError(f"reference_price is mid, mid_avg, far_touch or near_touch, not {reference_price!r}")
    rebate = (buy_v + sell_v) / tick * (rebate_bps / 10_000.0)
    buy_pnl = (ref_buy * buy_q - buy_v) / tick
    sell_pnl = (sell_v - ref_sell * sell_q) / tick
    bs = buy_pnl + sell_pnl
    inv_pnl = inv_prev * (mid1 - mid0) / tick
    pv = cash / tick + inv * ref / tick
    spooner = bs + rebate + inv_pnl
    asym = spooner - torch.clamp(eta * inv_pnl, min=0.0)
    table = {
        "portfolio_value": lambda: pv,
        "delta_portfolio_value": lambda: pv - (pv_prev if pv_prev is not None else pv),
        "buy_sell_pnl": lambda: bs,
        "spooner": lambda: spooner,
        "spooner_damped": lambda: spooner - eta * inv_pnl,
        "spooner_asym_damped": lambda: asym,
        "spooner_asym_damped2": lambda: bs + rebate + gamma * (inv_pnl - torch.clamp(eta * inv_pnl, min=0.0)),
        "spooner_scaled": lambda: bs + rebate + eta * (inv_pnl - (1.0 - eta) * torch.clamp(inv_pnl, min=0.0)),
        "complex": lambda: asym - lam * (inv - inv_prev).abs(),
        "zero_inv": lambda: -inv.abs(),
    }
    if name not in table:
        raise ValueError(f"unknown market-making reward {name!r}; one of {MM_REWARDS}")
    return table[name](), pv


INV_PENALTIES = ("none", "linear", "quadratic", "threshold", "exp4")


def inventory_penalty(kind: str, inv: torch.Tensor, weight: float, size: int, threshold: float = 10.0) -> torch.Tensor:
    """Inventory penalty in quote-size units q = inv / size (the reference's options,
    ``mm_env.py:2435-2456``): linear -w|q|, quadratic -w q^2, threshold -w q^2 only where
    |q| > ``threshold``, exp4 -w exp(4 q)."""
    q = inv.double() / size
    if kind == "none":
        return torch.zeros_like(q)
    if kind == "linear":
        return -weight * q.abs()
    if kind == "quadratic":
        return -weight * q * q
    if kind == "threshold":
        return torch.where(q.abs() > threshold, -weight * q * q, torch.zeros_like(q))
    if kind == "exp4":
        return -weight * torch.exp(4.0 * q)
    raise ValueError(f"inv_penalty is one of {INV_PENALTIES}, not {kind!r}")


UNWIND_PRICES = ("none", "mid", "mid_avg", "far_touch")


def unwind_fill(kind: str, inv: torch.Tensor, mid0, mid1, best_bid, best_ask, tick: int, penalty_ticks: int = 0):
    """The artificial end-of-episode trade that flattens ``inv`` (``mm_env.py:2206-2246``):
    (buy_q, buy_v, sell_q, sell_v) of one fill of |inv| shares at the unwind price -- the
    last mid, the step's average mid (here the mean of the mids before and after the step)
    or the far touch -- moved ``penalty_ticks`` against the agent."""
    zero = torch.zeros_like(inv)
    if kind == "none":
        return zero, zero, zero, zero
    if kind == "mid":
        p = mid1.long()
    elif kind == "mid_avg":
        p = (mid0.long() + mid1.long()) // 2
    elif kind == "far_touch":
        p = torch.where(inv > 0, best_bid.long(), best_ask.long())
    else:
        raise ValueError(f"unwind_price is one of {UNWIND_PRICES}, not {kind!r}")
    p = torch.where(inv > 0, p - penalty_ticks * tick, p + penalty_ticks * tick)
    sell_q = inv.clamp(min=0)
    buy_q = (-inv).clamp(min=0)
    return buy_q, buy_q * p, sell_q, sell_q * p


EXEC_SIZES = (0, 50, 100, 200, 400)
EXEC_QUANTS = ((0, 0), (1, 0), (0, 1), (1, 1), (2, 0), (0, 2))
EXEC_1MSG = ((0, 0), (1, 1), (2, 1), (1, 0), (2, 0))          # (size multiple, aggressive)
# the 13-action ladder (exec_env.py:838-932): nothing, then the far touch / the mid / the near
# touch / one level behind it at 1, 2 and 5 clips -- (level, multiple)
EXEC_COMPLEX = ((0, 0),) + tuple((lvl, m) for m in (1, 2, 5) for lvl in range(4))


def exec_orders(space: str, action: torch.Tensor, st: Dict[str, torch.Tensor], remaining: torch.Tensor,
                clip: int, steps_left, sell, tick: int):
    """(resting orders (n, K, 3), marketable qty (n,)) of an executor working ``remaining``
    shares; the far touch is the price that trades now (the ask for a buyer).  ``sell`` is a
    bool or a per-environment bool tensor; ``steps_left`` an int or a per-environment tensor
    (this step included)."""
    bb, ba, mid = st["best_bid"], st["best_ask"], st["mid"]
    sell = torch.as_tensor(sell, dtype=torch.bool).expand(mid.shape)
    near = torch.where(sell, ba, bb)
    side = torch.where(sell, -1, 1)
    behind = near - side * tick                     # one tick less aggressive than the near touch
    one, zero = torch.ones_like(mid), torch.zeros_like(mid)
    a = action.long()
    take = zero.clone()
    # the mid on the tick grid: floored for a buyer, rounded up for a seller
    mid_px = torch.where(sell, -((-mid) // tick) * tick, (mid // tick) * tick)
    if space == "sizes":
        take = torch.tensor(EXEC_SIZES)[a]
        orders = _rows((zero, zero, zero))
    elif space == "fixed_quants":
        t = torch.tensor(EXEC_QUANTS)[a]
        take = t[:, 0] * clip
        orders = _rows((one * side, near, t[:, 1] * clip))
    elif space == "fixed_quants_1msg":
        t = torch.tensor(EXEC_1MSG)[a]
        q = t[:, 0] * clip
        take = torch.where(t[:, 1] == 1, q, zero)
        orders = _rows((one * side, near, torch.where(t[:, 1] == 1, zero, q)))
    elif space == "fixed_prices":
        take = a[:, 0] * clip
        orders = _rows((one * side, mid_px, a[:, 1] * clip), (one * side, near, a[:, 2] * clip),
                       (one * side, behind, a[:, 3] * clip))
    elif space == "fixed_quants_complex":
        t = torch.tensor(EXEC_COMPLEX)[a]
        lvl, q = t[:, 0], t[:, 1] * clip
        # an order larger than what is left sends all of it to the far touch
        over = q > remaining
        take = torch.where(over, remaining, torch.where(lvl == 0, q, zero))
        rest = torch.where(over | (lvl == 0), zero, q)
        price = torch.where(lvl == 1, mid_px, torch.where(lvl == 2, near, behind))
        orders = _rows((one * side, price, rest))
    elif space == "simplest_case":
        take = torch.where(a == 1, one * clip, zero)
        orders = _rows((zero, zero, zero))
    elif space == "twap":
        take = -(-remaining // torch.as_tensor(steps_left).clamp(min=1))
        orders = _rows((zero, zero, zero))
    else:
        raise ValueError(f"unknown execution action space {space!r}; one of {EXEC_ACTION_SPACES}")
    take = torch.minimum(take.long(), remaining)
    # resting orders never exceed what is left after the marketable part
    left = (remaining - take).clamp(min=0)
    cum = torch.cumsum(orders[..., 2], 1)
    orders[..., 2] = torch.clamp(torch.minimum(cum, left[:, None]) - (cum - orders[..., 2]), min=0)
    bad = (orders[..., 2] <= 0) | (orders[..., 1] <= 0) | (mid <= 0)[:, None]
    orders[bad] = 0
    return orders, take


def exec_reward(name: str, *, filled, value, market_q, market_v, arrival, target: int, sell, tick: int,
                lam: float = 1.0, remaining=None, mid_avg=None, scaling: float = 1.0):
    """Reward of the executor's fills of the step: ``filled`` shares for ``value`` (sum of
    price x qty); ``market_q`` / ``market_v`` the other traders' volume and value (VWAP).

    The reference's own rewards (``exec_env.py:1511-1758``, divided by ``scaling``, its
    reward_scaling_quo): ``normal`` = advantage over the other traders' VWAP plus ``lam`` x
    the drift of that VWAP from the arrival price, in ticks x shares (the VWAP falls back
    to the step's average mid ``mid_avg`` when nobody else traded); ``finish_fast`` =
    -(shares left after the step); ``simplest_case`` = the fills' price improvement over the
    arrival price, in price units x shares."""
    d = torch.float64
    filled, value, arrival = filled.to(d), value.to(d), arrival.to(d)
    sgn = torch.where(torch.as_tensor(sell, dtype=torch.bool).expand(filled.shape), -1.0, 1.0).to(d)
    if name == "normal":
        fb = (mid_avg if mid_avg is not None else arrival).to(d)
        vwap = torch.where(market_q > 0, market_v.to(d) / market_q.to(d).clamp(min=1), fb) // tick
        advantage = -sgn * (value / tick - vwap * filled)
        drift = -sgn * filled * (vwap - arrival // tick)
        return (advantage + lam * drift) / scaling
    if name == "finish_fast":
        return -remaining.to(d).abs() / scaling
    if name == "simplest_case":
        return -sgn * (value - arrival * filled) / scaling
    if name == "slippage":
        avg = value / filled.clamp(min=1)
        short = (avg - arrival) * sgn / tick
        return torch.where(filled > 0, -short * filled / target, torch.zeros_like(short))
    if name == "vwap":
        vwap = torch.where(market_q > 0, market_v.to(d) / market_q.to(d).clamp(min=1), arrival) / tick
        # advantage: the executor's proceeds against the market VWAP (a seller gains above it)
        advantage = -sgn * (value / tick - vwap * filled)
        drift = -sgn * filled * (vwap - arrival / tick)
        return (advantage + lam * drift) / target
    raise ValueError(f"unknown execution reward {name!r}; one of {EXEC_REWARDS}")


def touch(l2: torch.Tensor, tick: int):
    """(best_bid, best_ask, tick-floored mid) of (n, 4L) L2 rows; zeros where a side is empty."""
    ap, bp = l2[:, 0].long(), l2[:, 2].long()
    ok = (ap < 2**31 - 1) & (bp > -(2**31 - 1)) & (ap > 0) & (bp > 0)
    z = torch.zeros_like(ap)
    mid = torch.where(ok, (ap + bp) // 2 // tick * tick, z)
    return torch.where(ok, bp, z), torch.where(ok, ap, z), mid

