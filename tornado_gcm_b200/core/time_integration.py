"""Implicit-explicit (IMEX) time steppers on pytrees of tensors.

API and schemes follow reference ``core/time_integration.py:76-424``:
forward/backward Euler, Crank-Nicolson RK2, low-storage CN-RK3/RK4
(Williamson; Carpenter-Kennedy), the generic IMEX Runge-Kutta driver with
an explicit Butcher tableau and SIL3 (Whitaker & Kar 2013), step filters
and trajectory helpers.  These are the reference-semantics (CPU/oracle)
steppers; the fused GPU stepper in :mod:`tornado_gcm_b200.ops.dycore`
implements the same SIL3 tableau with the stage algebra folded into the
implicit-solve kernel.
"""

from __future__ import annotations

import dataclasses
from typing import Any, Callable, Optional, Sequence, Union

import torch

from tornado_gcm_b200.core import filtering

PyTreeState = Any
TimeStepFn = Callable[[PyTreeState], PyTreeState]


def tree_map(fn, *trees):
    first = trees[0]
    if isinstance(first, torch.Tensor):
        return fn(*trees)
    if isinstance(first, dict):
        return {k: tree_map(fn, *[t[k] for t in trees]) for k in first}
    if isinstance(first, (list, tuple)):
        return type(first)(tree_map(fn, *[t[i] for t in trees]) for i in range(len(first)))
    if dataclasses.is_dataclass(first) and not isinstance(first, type):
        updates = {}
        for f in dataclasses.fields(first):
            v = getattr(first, f.name)
            if isinstance(v, (torch.Tensor, dict, list, tuple)) or (
                dataclasses.is_dataclass(v) and not isinstance(v, type)
            ):
                updates[f.name] = tree_map(fn, *[getattr(t, f.name) for t in trees])
        return dataclasses.replace(first, **updates)
    return first


def tree_add(a, b):
    return tree_map(torch.add, a, b)


def tree_scale(tree, c: float):
    return tree_map(lambda x: x * c, tree)


def tree_axpy(y, a: float, x):
    """y + a·x on pytrees."""
    return tree_map(lambda yi, xi: yi + a * xi, y, x)


def tree_neg(tree):
    return tree_map(torch.neg, tree)


class ExplicitODE:
    def explicit_terms(self, state):
        raise NotImplementedError

    @classmethod
    def from_functions(cls, explicit_terms):
        ode = cls()
        ode.explicit_terms = explicit_terms
        return ode


class ImplicitExplicitODE:
    """∂x/∂t = F(x) + G(x): explicit F, implicit G, and (I - ηG)⁻¹."""

    def explicit_terms(self, state):
        raise NotImplementedError

    def implicit_terms(self, state):
        raise NotImplementedError

    def implicit_inverse(self, state, step_size: float):
        raise NotImplementedError

    @classmethod
    def from_functions(cls, explicit_terms, implicit_terms, implicit_inverse):
        ode = cls()
        ode.explicit_terms = explicit_terms
        ode.implicit_terms = implicit_terms
        ode.implicit_inverse = implicit_inverse
        return ode


@dataclasses.dataclass
class TimeReversedImExODE(ImplicitExplicitODE):
    forward_eq: ImplicitExplicitODE

    def explicit_terms(self, state):
        return tree_neg(self.forward_eq.explicit_terms(state))

    def implicit_terms(self, state):
        return tree_neg(self.forward_eq.implicit_terms(state))

    def implicit_inverse(self, state, step_size):
        return self.forward_eq.implicit_inverse(state, -step_size)


def compose_equations(equations: Sequence[Union[ImplicitExplicitODE, ExplicitODE]]) -> ImplicitExplicitODE:
    imex = [e for e in equations if isinstance(e, ImplicitExplicitODE)]
    if len(imex) != 1:
        raise ValueError(f"Expected exactly 1 ImplicitExplicitODE, got {len(imex)}")
    (imex_eq,) = imex

    def explicit_fn(x):
        out = None
        for eq in equations:
            t = eq.explicit_terms(x)
            out = t if out is None else tree_add(out, t)
        return out

    return ImplicitExplicitODE.from_functions(explicit_fn, imex_eq.implicit_terms, imex_eq.implicit_inverse)


def backward_forward_euler(equation: ImplicitExplicitODE, time_step: float) -> TimeStepFn:
    def step_fn(u0):
        return equation.implicit_inverse(tree_axpy(u0, time_step, equation.explicit_terms(u0)), time_step)
    return step_fn


def crank_nicolson_rk2(equation: ImplicitExplicitODE, time_step: float) -> TimeStepFn:
    dt = time_step

    def step_fn(u0):
        g = tree_axpy(u0, 0.5 * dt, equation.implicit_terms(u0))
        h1 = equation.explicit_terms(u0)
        u1 = equation.implicit_inverse(tree_axpy(g, dt, h1), 0.5 * dt)
        h2 = tree_map(lambda a, b: 0.5 * (a + b), equation.explicit_terms(u1), h1)
        return equation.implicit_inverse(tree_axpy(g, dt, h2), 0.5 * dt)
    return step_fn


def low_storage_runge_kutta_crank_nicolson(alphas, betas, gammas, equation, time_step) -> TimeStepFn:
    dt = time_step
    if len(alphas) - 1 != len(betas) or len(betas) != len(gammas):
        raise ValueError("RK coefficient lengths don't match")

    def step_fn(u):
        h = None
        for k in range(len(betas)):
            fu = equation.explicit_terms(u)
            h = fu if h is None else tree_axpy(fu, betas[k], h)
            mu = 0.5 * dt * (alphas[k + 1] - alphas[k])
            rhs = tree_axpy(tree_axpy(u, gammas[k] * dt, h), mu, equation.implicit_terms(u))
            u = equation.implicit_inverse(rhs, mu)
        return u
    return step_fn


def crank_nicolson_rk3(equation, time_step) -> TimeStepFn:
    return low_storage_runge_kutta_crank_nicolson(
        alphas=[0, 1 / 3, 3 / 4, 1], betas=[0, -5 / 9, -153 / 128], gammas=[1 / 3, 15 / 16, 8 / 15],
        equation=equation, time_step=time_step)


def crank_nicolson_rk4(equation, time_step) -> TimeStepFn:
    return low_storage_runge_kutta_crank_nicolson(
        alphas=[0, 0.1496590219993, 0.3704009573644, 0.6222557631345, 0.9582821306748, 1],
        betas=[0, -0.4178904745, -1.192151694643, -1.697784692471, -1.514183444257],
        gammas=[0.1496590219993, 0.3792103129999, 0.8229550293869, 0.6994504559488, 0.1530572479681],
        equation=equation, time_step=time_step)


@dataclasses.dataclass
class ImExButcherTableau:
    a_ex: Sequence[Sequence[float]]
    a_im: Sequence[Sequence[float]]
    b_ex: Sequence[float]
    b_im: Sequence[float]


SIL3_TABLEAU = ImExButcherTableau(
    a_ex=[[1 / 3], [1 / 6, 1 / 2], [1 / 2, -1 / 2, 1]],
    a_im=[[1 / 6, 1 / 6], [1 / 3, 0, 1 / 3], [3 / 8, 0, 3 / 8, 1 / 4]],
    b_ex=[1 / 2, -1 / 2, 1, 0],
    b_im=[3 / 8, 0, 3 / 8, 1 / 4],
)


@dataclasses.dataclass(frozen=True)
class _StagePlan:
    """One stage of a compiled IMEX-RK tableau.

    ``terms``: the (weight, kind, index) products added to y0 to form the stage's
    right-hand side, kind ``"F"`` (explicit tendency of stage index) or ``"G"``
    (implicit tendency); ``eta``: the implicit weight of the stage's solve;
    ``keep``: which of this stage's tendencies a later stage or the final
    combination reads (the others are never evaluated).
    """

    terms: tuple
    eta: float
    keep: frozenset


def compile_imex_tableau(tableau: ImExButcherTableau, dt: float) -> tuple:
    """(stage plans, final terms) of ``tableau`` at step ``dt``.

    The tableau is turned into a small program once: row ``i - 1`` of ``a_ex`` /
    ``a_im`` gives stage i's right-hand side (zero weights dropped), the diagonal
    entry ``a_im[i - 1][i]`` its implicit weight, and a liveness pass from the
    last combination backwards marks the tendencies that are read at all.
    """
    a_ex, a_im, b_ex, b_im = tableau.a_ex, tableau.a_im, tableau.b_ex, tableau.b_im
    n = len(b_ex)

    def products(row_ex, row_im, width):
        out = []
        for j in range(width):
            if j < len(row_ex) and row_ex[j]:
                out.append((dt * row_ex[j], "F", j))
            if j < len(row_im) and row_im[j]:
                out.append((dt * row_im[j], "G", j))
        return tuple(out)

    rhs = [()] + [products(a_ex[i - 1], a_im[i - 1], i) for i in range(1, n)]
    etas = [0.0] + [dt * a_im[i - 1][i] for i in range(1, n)]
    final = products(b_ex, b_im, n)
    live = {(k, j) for _, k, j in final}
    plans = [None] * n
    for i in range(n - 1, -1, -1):
        plans[i] = _StagePlan(rhs[i], etas[i], frozenset(k for k in ("F", "G") if (k, i) in live))
        live |= {(k, j) for _, k, j in rhs[i]}
    return tuple(plans), final


def imex_runge_kutta(tableau: ImExButcherTableau, equation: ImplicitExplicitODE, time_step: float,
                     step_hook: Optional[Callable[[int, Any], None]] = None) -> TimeStepFn:
    """Generic IMEX-RK: y_i = (I - dt a_im[i,i] G)^{-1}(y0 + dt Σ_j<i a_ex F_j + a_im G_j).

    Stage 0 is y0 itself; the step returns y0 + dt Σ_j (b_ex F_j + b_im G_j).
    Tendencies that no later combination reads are not evaluated.
    """
    plans, final = compile_imex_tableau(tableau, time_step)
    tendency = {"F": equation.explicit_terms, "G": equation.implicit_terms}

    def combine(y0, terms, tend):
        y = y0
        for w, kind, j in terms:
            y = tree_axpy(y, w, tend[kind, j])
        return y

    def step_fn(y0):
        tend = {}
        for i, plan in enumerate(plans):
            if i == 0:
                y_i = y0
            else:
                y_i = equation.implicit_inverse(combine(y0, plan.terms, tend), plan.eta)
                if step_hook is not None:
                    step_hook(i, y_i)
            for kind in ("F", "G"):
                if kind in plan.keep:
                    tend[kind, i] = tendency[kind](y_i)
        return combine(y0, final, tend)
    return step_fn


def imex_rk_sil3(equation: ImplicitExplicitODE, time_step: float,
                 step_hook: Optional[Callable[[int, Any], None]] = None) -> TimeStepFn:
    return imex_runge_kutta(SIL3_TABLEAU, equation, time_step, step_hook)


def runge_kutta_step_filter(state_filter):
    def _filter(u, u_next):
        return state_filter(u_next)
    return _filter


def exponential_step_filter(grid, dt: float, tau: float = 0.010938, order: int = 18, cutoff: float = 0):
    filt = filtering.exponential_filter(grid, dt / tau, order, cutoff)
    return runge_kutta_step_filter(lambda s: tree_map(filt, s))


def horizontal_diffusion_step_filter(grid, dt: float, tau: float, order: int = 1):
    """∇^(2·order) diffusion as a step filter: the truncation wavenumber decays by
    exp(-dt / tau) per step, lower ones by (λ_l / λ_max)^order of that rate.

    ``filtering.horizontal_diffusion_filter`` applies exp(scale · (-λ)^order)
    (reference ``core/filtering.py:55-78``), so a damping filter takes a negative
    scale.  Reference ``core/time_integration.py:358-368`` passes +dt / (τ λ_max^order),
    which grows the truncation wavenumber by exp(dt/τ) per step: with the 0.7°
    time scales that anti-diffusion made random-init rollouts blow up after
    about nine simulated hours.
    """
    eig = grid.laplacian_eigenvalues
    scale = -dt / (tau * abs(eig[-1]) ** order)
    filt = filtering.horizontal_diffusion_filter(grid, scale, order)
    return runge_kutta_step_filter(lambda s: tree_map(filt, s))


def step_with_filters(step_fn: TimeStepFn, filters) -> TimeStepFn:
    def _step(u):
        u_next = step_fn(u)
        for f in filters:
            u_next = f(u, u_next)
        return u_next
    return _step


def repeated(fn: TimeStepFn, steps: int) -> TimeStepFn:
    if steps == 1:
        return fn

    def f_rep(x):
        for _ in range(steps):
            x = fn(x)
        return x
    return f_rep


def trajectory_from_step(step_fn: TimeStepFn, outer_steps: int, inner_steps: int, *,
                         start_with_input: bool = False, post_process_fn=lambda x: x):
    if inner_steps != 1:
        step_fn = repeated(step_fn, inner_steps)

    def multistep(x):
        traj = []
        for _ in range(outer_steps):
            if start_with_input:
                traj.append(post_process_fn(x))
            x = step_fn(x)
            if not start_with_input:
                traj.append(post_process_fn(x))
        return x, traj
    return multistep
