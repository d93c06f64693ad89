"""Selector -> execution entry: plan_fft / execute_fft_plan / run_fft.

Drop-in B200 counterpart of the reference's ``src/xpu/entry.py``:

1. semantics are validated before any table query or launch (ValueError);
2. the frozen B200 table is queried (``selector.select``), an exact-shape
   composition entry outranks it for c2c/forward/backward;
3. abstain / undispatchable falls back to M0 (``fft_dit`` / ``fft_dif``, batch
   > 1: the M4 stage flow, ``folded`` variant) with the reason recorded;
4. ``execute_fft_plan`` checks the input against the plan (TypeError /
   ValueError before any launch) and runs the whole plan -- inverse
   conjugation, norm epilogue and the real-transform wrapper included -- as
   one native plan of libbfft.so on the tensor's current stream.

``ExecutionPlan`` fields, reason templates and fallback semantics are the
reference's (entry.py:105-426).  On B200 the inverse conjugation and the norm
scale are fused into the first and last kernel instead of separate passes,
and the real pack is a zero-copy reinterpretation of the float32 input.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

from .composition import composition_select
from .config import NORMALIZATIONS, TRANSFORM_DIRECTIONS, TRANSFORM_TYPES
from .selector import Selection, find_entry, load_table, select

DEFAULT_BLOCK = 1024
SUPPORTED_DIRECTIONS = ("dit", "dif")
SUPPORTED_PRECISIONS = ("fp32",)
SUPPORTED_TRANSFORMS = TRANSFORM_TYPES
SUPPORTED_TRANSFORM_DIRECTIONS = TRANSFORM_DIRECTIONS
SUPPORTED_NORMS = NORMALIZATIONS
REAL_COMPAT_MARK = "packed-c2c-compat"
REAL_FLOW_MARK = "dedicated-half-spectrum"
_SUPPORTED_DTYPES = {"fp32": "complex64"}


def norm_scale(n: int, transform_direction: str, norm: str) -> float:
    """Epilogue scale of one (direction, norm) pair, torch.fft semantics.

    ========= ========= =========
    norm      forward   inverse
    ========= ========= =========
    none      1         1
    forward   1/N       1
    backward  1         1/N
    ortho     1/sqrt N  1/sqrt N
    ========= ========= =========
    """
    if transform_direction not in SUPPORTED_TRANSFORM_DIRECTIONS:
        raise ValueError(f"bad transform_direction {transform_direction!r}")
    if norm not in SUPPORTED_NORMS:
        raise ValueError(f"bad norm {norm!r}")
    if norm == "ortho":
        return 1.0 / math.sqrt(n)
    if (norm, transform_direction) in (("forward", "forward"), ("backward", "inverse")):
        return 1.0 / n
    return 1.0


@dataclass(frozen=True)
class ExecutionPlan:
    """What runs for one shape under the frozen table (entry.py:105-128)."""

    n: int
    batch: int
    direction: str
    precision: str
    selection_source: str  # "table" | "abstain" | "composition"
    reason: str
    fallback: bool
    executed: str
    block: int | None = None
    flow_id: str | None = None
    flow_realization: str | None = None
    processing_unit: str | None = None
    params: dict = field(default_factory=dict)
    transform_type: str = "c2c"
    transform_direction: str = "forward"
    norm: str = "backward"

    def as_report(self) -> "ExecutionReport":
        return ExecutionReport(**self.__dict__)


@dataclass(frozen=True)
class ExecutionReport(ExecutionPlan):
    """ExecutionPlan plus the observation that it was carried out."""


def _validate_semantics(direction: str, precision: str, transform_type: str = "c2c",
                        transform_direction: str = "forward", norm: str = "backward") -> None:
    """Reject unsupported semantics before any table query or launch."""
    if direction not in SUPPORTED_DIRECTIONS:
        raise ValueError(f"unsupported direction {direction!r}; supported: {SUPPORTED_DIRECTIONS} "
                         "(the decomposition); unknown directions must not fall back to a different transform")
    if precision not in SUPPORTED_PRECISIONS:
        raise ValueError(f"unsupported precision {precision!r}; supported: {SUPPORTED_PRECISIONS}")
    if transform_type not in SUPPORTED_TRANSFORMS:
        raise ValueError(f"unsupported transform_type {transform_type!r}; supported: {SUPPORTED_TRANSFORMS}; "
                         "unknown transforms must not fall back to a different one")
    if transform_direction not in SUPPORTED_TRANSFORM_DIRECTIONS:
        raise ValueError(f"unsupported transform_direction {transform_direction!r}; "
                         f"supports {SUPPORTED_TRANSFORM_DIRECTIONS}")
    if norm not in SUPPORTED_NORMS:
        raise ValueError(f"unsupported norm {norm!r}; supports {SUPPORTED_NORMS}")
    if transform_type == "r2c" and transform_direction != "forward":
        raise ValueError(f"r2c is a forward transform; got transform_direction={transform_direction!r}")
    if transform_type == "c2r" and transform_direction != "inverse":
        raise ValueError(f"c2r is an inverse transform; got transform_direction={transform_direction!r}")


def _m0_name(direction: str, batch: int) -> str:
    if batch > 1:
        return "fft_dit_batch" if direction == "dit" else "fft_dif_batch"
    return "fft_dit" if direction == "dit" else "fft_dif"


def _m0_plan(n, batch, direction, precision, reason, fallback, block=DEFAULT_BLOCK,
             transform_type="c2c", transform_direction="forward", norm="backward") -> ExecutionPlan:
    return ExecutionPlan(
        n=n, batch=batch, direction=direction, precision=precision,
        selection_source="abstain" if fallback else "table", reason=reason, fallback=fallback,
        executed=_m0_name(direction, batch), block=block, flow_id="baseline-global-stage",
        flow_realization="global-stage", processing_unit="radix2-scalar",
        params=({"variant": "folded", "batch": batch} if batch > 1 else {}),
        transform_type=transform_type, transform_direction=transform_direction, norm=norm)


def _dispatch(sel: Selection) -> str | None:
    """Runner name for a table selection, or None when nothing lowers it
    (entry.py:197-225)."""
    key = (sel.flow_realization, sel.processing_unit, sel.direction)
    batched = sel.batch != 1
    table = {
        ("global-stage", "radix2-scalar", "dit"): ("fft_dit", "fft_dit_batch"),
        ("global-stage", "radix2-scalar", "dif"): ("fft_dif", "fft_dif_batch"),
        ("global-stage", "radix4-scalar", "dit"): ("fft_dit_radix4", "fft_dit_radix4_batch"),
        ("global-stage", "radix4-scalar", "dif"): ("fft_dif_radix4", "fft_dif_radix4_batch"),
        ("matrix-resident", "dense-dot-fft64", "dit"): ("fft_dit_matrix", "fft_dit_matrix_batch"),
        ("matrix-resident", "dense-dot-fft64", "dif"): ("fft_dif_matrix", "fft_dif_matrix_batch"),
    }
    if key in table:
        return table[key][1 if batched else 0]
    if batched:
        return None
    return {
        ("fused-inplace", "radix2-scalar", "dit"): "fft_dit_fused",
        ("grouped-boundary", "composite-linear-map", "dit"): "fft_dit_grouped",
        ("grouped-boundary", "composite-linear-map", "dif"): "fft_dif_grouped",
    }.get(key)


def _composition_plan(comp: dict, n: int, batch: int, direction: str, precision: str,
                      transform_direction: str, norm: str) -> ExecutionPlan:
    ev = comp["evidence"]
    reason = (f"composition {comp['flow_id']} (exact shape, {comp['guard_pct']:.1f}% >= {2.0}% guard vs "
              f"{comp.get('incumbent_flow', 'incumbent')}; p50={ev['p50_ms']:.4f}ms over {ev['sessions']} "
              f"sessions + confirmation, err_max={ev['err_max']:g}): {comp['reason']}")
    return ExecutionPlan(
        n=n, batch=batch, direction=direction, precision=precision, selection_source="composition",
        reason=reason, fallback=False, executed="run_hybrid", block=None, flow_id=comp["flow_id"],
        flow_realization=comp["flow_realization"], processing_unit=comp["processing_unit"],
        params={"flow_kind": "composition", "tile": comp["tile"], "core": comp["core"],
                "contract_id": comp.get("contract_id") or comp.get("_contract_id"),
                "composition_guard_pct": comp["guard_pct"], "evidence_artifact": ev["artifact"]},
        transform_type="c2c", transform_direction=transform_direction, norm=norm)


def _with_compat(plan: ExecutionPlan, compat: dict) -> ExecutionPlan:
    params = dict(plan.params or {})
    params.update(compat)
    return ExecutionPlan(**{**plan.__dict__, "params": params})


def _entry_block(table: dict, sel: Selection) -> int:
    e = find_entry(table, sel.n, sel.batch, sel.direction, sel.transform_type,
                   sel.transform_direction, sel.normalization)
    if e is None:
        return DEFAULT_BLOCK
    return int(e.get("incumbent_block") or e.get("block") or DEFAULT_BLOCK)


def plan_fft(direction: str, n: int, batch: int = 1, precision: str = "fp32",
             profile_hash: str | None = None, table: dict | None = None,
             env_hash: str | None = "auto", transform_type: str = "c2c",
             transform_direction: str | None = None, norm: str = "backward") -> ExecutionPlan:
    """Resolve the frozen table onto a concrete plan (host-only, no torch).

    Unsupported semantics raise ValueError before the table query.
    ``profile_hash=None``, an unknown or stale environment, or a shape outside
    the measured matrix falls back to M0 with the reason; a table entry no
    runner lowers falls back to M0 with ``"no lowering for ...; M0 fallback"``.
    """
    if transform_direction is None:
        transform_direction = "inverse" if transform_type == "c2r" else "forward"
    _validate_semantics(direction, precision, transform_type, transform_direction, norm)
    if transform_type == "c2c":
        comp = composition_select(direction, n, batch=batch, precision=precision,
                                  profile_hash=profile_hash, env_hash=env_hash,
                                  transform_type=transform_type,
                                  transform_direction=transform_direction, normalization=norm)
        if comp is not None:
            return _composition_plan(comp, n, batch, direction, precision, transform_direction, norm)
    table = table if table is not None else load_table()
    sel = select(direction, n, batch=batch, precision=precision, profile_hash=profile_hash,
                 table=table, env_hash=env_hash, transform_type=transform_type,
                 transform_direction=transform_direction, normalization=norm)
    compat = {"real_compat": REAL_COMPAT_MARK} if transform_type in ("r2c", "c2r") else {}
    if not sel.selected:
        plan = _m0_plan(n, batch, direction, precision, sel.reason, True, block=_entry_block(table, sel),
                        transform_type=transform_type, transform_direction=transform_direction, norm=norm)
        return _with_compat(plan, compat) if compat else plan
    name = sel.executed or _dispatch(sel)
    if name is None:
        plan = _m0_plan(n, batch, direction, precision,
                        f"no lowering for {sel.flow_realization}/{sel.processing_unit} "
                        f"direction={direction} batch={batch}; M0 fallback",
                        True, block=_entry_block(table, sel), transform_type=transform_type,
                        transform_direction=transform_direction, norm=norm)
        return _with_compat(plan, compat) if compat else plan
    params = dict(sel.params or {})
    if sel.entry_tier == "previous-fallback":
        params["previous_fallback"] = True
    if params.get("real_flow"):
        from .semantic import family_allows

        if not family_allows(transform_type, params["real_flow"]):
            raise ValueError(f"real_flow {params['real_flow']!r} not in the {transform_type} family")
        params["real_compat"] = REAL_FLOW_MARK
    else:
        params.update(compat)
    return ExecutionPlan(
        n=n, batch=batch, direction=direction, precision=precision, selection_source="table",
        reason=sel.reason, fallback=False, executed=name, block=sel.block, flow_id=sel.flow_id,
        flow_realization=sel.flow_realization, processing_unit=sel.processing_unit, params=params,
        transform_type=transform_type, transform_direction=transform_direction, norm=norm)


def _expected_input_n(plan: ExecutionPlan) -> int:
    return plan.n // 2 + 1 if plan.transform_type == "c2r" else plan.n


def _check_plan_input(plan: ExecutionPlan, shape, dtype_name: str) -> None:
    """Host-testable shape / dtype contract of plan-reuse execution (entry.py:467-498)."""
    want = "float32" if plan.transform_type == "r2c" else _SUPPORTED_DTYPES.get(plan.precision, "complex64")
    if dtype_name != want:
        raise TypeError(f"x must be {want} for transform_type={plan.transform_type} "
                        f"precision={plan.precision}, got {dtype_name}")
    shape = tuple(int(s) for s in shape)
    n_expect = _expected_input_n(plan)
    if plan.batch == 1:
        if len(shape) != 1 or shape[0] != n_expect:
            raise ValueError(f"plan expects rank-1 x with N={n_expect} (batch=1, "
                             f"transform_type={plan.transform_type}); got shape {shape}")
    elif len(shape) != 2 or shape != (plan.batch, n_expect):
        raise ValueError(f"plan expects x shape ({plan.batch}, {n_expect}); got shape {shape}")


def _runner_knobs(plan: ExecutionPlan) -> dict:
    """The runner arguments the reference's _invoke passes (entry.py:429-456)."""
    p = plan.params or {}
    name = plan.executed
    block = int(plan.block or DEFAULT_BLOCK)
    k: dict = {"block": block}
    if name == "fft_dit_fused":
        k["tile"] = int(p.get("tile", 64))
    elif name in ("fft_dit_matrix", "fft_dif_matrix", "fft_dit_matrix_batch", "fft_dif_matrix_batch"):
        k["tile"] = int(p.get("tile", 64))
        k["rows"] = int(p.get("rows", 8))
        if name.endswith("_batch"):
            k["variant"] = str(p.get("variant", "spread"))
    elif name in ("fft_dit_radix4_batch", "fft_dif_radix4_batch"):
        k["variant"] = str(p.get("variant", "spread"))
    elif name in ("fft_dit_grouped", "fft_dif_grouped"):
        k.update(tile=int(p.get("tile", 64)), rows=int(p.get("rows", 8)), glog=int(p.get("glog", 2)),
                 maxp=int(p.get("maxp", 4096)), cells=int(p.get("cells", 1)))
    elif name in ("fft_dit_batch", "fft_dif_batch"):
        k["variant"] = str(p.get("variant", "folded"))
    elif name == "run_hybrid":
        k["tile"] = int(p.get("tile", 64))
    elif name not in ("fft_dit", "fft_dif", "fft_dit_radix4", "fft_dif_radix4"):
        raise AssertionError(f"unmapped runner function {name!r}")
    return k


def native_plan_for(plan: ExecutionPlan, device: int):
    """libbfft plan executing ``plan`` on ``device`` (cached per plan key)."""
    from . import _lib
    from .runner import native_plan

    knobs = _runner_knobs(plan)
    real_flow = bool((plan.params or {}).get("real_flow"))
    variant = knobs.pop("variant", "spread")
    return native_plan(plan.executed, plan.direction, plan.n, plan.batch, device,
                       transform_type=plan.transform_type,
                       transform_direction=plan.transform_direction, norm=plan.norm,
                       real_flow=real_flow and plan.transform_type != "c2c", variant=variant, **knobs) \
        if plan.executed in _lib.RUNNER_IDS else None


# Plans already validated on a device: id(plan), device -> (weakref to the plan,
# native plan, x shape, x dtype, out shape, out dtype).  A hit skips the
# plan-level checks and the plan lookup; x is still checked on every call.
_VALIDATED: dict = {}


def _remember(plan: ExecutionPlan, dev: int, native, x, out) -> None:
    import weakref

    key = (id(plan), dev)

    def _drop(ref, key=key):
        ent = _VALIDATED.get(key)
        if ent is not None and ent[0] is ref:
            _VALIDATED.pop(key, None)

    try:
        ref = weakref.ref(plan, _drop)
    except TypeError:
        return
    _VALIDATED[key] = (ref, native, tuple(x.shape), x.dtype, tuple(out.shape), out.dtype)


def execute_fft_plan(plan: ExecutionPlan, x):
    """Execute a resolved plan without re-querying the table (plan reuse).

    ``x`` must sit on a CUDA device with the plan's shape and dtype (checked
    before any launch).  Output is a fresh tensor: complex64 (c2c, r2c half
    spectrum) or float32 (c2r).
    """
    import torch

    from . import _lib
    from .ledger import _ACTIVE, phase
    from .runner import execute_native

    if _ACTIVE.get() is None and type(x) is torch.Tensor and x.is_cuda:
        dev = x.device.index if x.device.index is not None else torch.cuda.current_device()
        ent = _VALIDATED.get((id(plan), dev))
        if ent is not None and ent[0]() is plan and tuple(x.shape) == ent[2] and x.dtype == ent[3] \
                and x.is_contiguous() and x.data_ptr() % 8 == 0:
            return execute_native(ent[1], x, torch.empty(ent[4], dtype=ent[5], device=x.device))

    with phase("plan-validate"):
        if not isinstance(x, torch.Tensor):
            raise TypeError(f"x must be a torch.Tensor, got {type(x).__name__}")
        _check_plan_input(plan, tuple(x.shape), str(x.dtype).split(".")[-1])
        if plan.transform_type not in SUPPORTED_TRANSFORMS:
            raise ValueError(f"plan transform_type {plan.transform_type!r} not supported")
        if plan.transform_direction not in SUPPORTED_TRANSFORM_DIRECTIONS:
            raise ValueError(f"plan transform_direction {plan.transform_direction!r} not supported")
        if plan.norm not in SUPPORTED_NORMS:
            raise ValueError(f"plan norm {plan.norm!r} not supported")
        if plan.params.get("flow_kind") == "composition" and plan.transform_type != "c2c":
            raise ValueError(f"composition plans support transform_type='c2c' only, got {plan.transform_type!r}")
        real_flow = plan.params.get("real_flow")
        if real_flow is not None:
            from .semantic import family_allows

            if plan.transform_type not in ("r2c", "c2r"):
                raise ValueError(f"real_flow plans support transform_type r2c/c2r only, got {plan.transform_type!r}")
            if not family_allows(plan.transform_type, real_flow):
                raise ValueError(f"real_flow {real_flow!r} not in the {plan.transform_type} family")
        if x.device.type != "cuda":
            raise ValueError(f"x must be on a CUDA device, got device={x.device}")
        if not x.is_contiguous():
            raise ValueError("x must be contiguous")
        if x.data_ptr() % 8:
            raise ValueError("x must start on an 8-byte boundary (complex64 / float32 pairs)")
        if plan.executed not in _lib.RUNNER_IDS:
            raise AssertionError(f"unmapped runner function {plan.executed!r}")
    dev = x.device.index if x.device.index is not None else torch.cuda.current_device()
    with phase("core-invoke"):
        native = native_plan_for(plan, dev)
        if plan.transform_type == "r2c":
            out = torch.empty((*x.shape[:-1], plan.n // 2 + 1), dtype=torch.complex64, device=x.device)
        elif plan.transform_type == "c2r":
            out = torch.empty((*x.shape[:-1], plan.n), dtype=torch.float32, device=x.device)
        else:
            out = torch.empty_like(x)
        _remember(plan, dev, native, x, out)
        return execute_native(native, x, out)


def run_fft(x, direction: str, *, batch: int | None = None, precision: str = "fp32",
            profile_hash: str | None = None, table: dict | None = None, transform_type: str = "c2c",
            transform_direction: str | None = None, norm: str = "backward"):
    """One-shot plan + execute; returns ``(y, ExecutionReport)`` (entry.py:699-758).
    A rank-2 ``(1, N)`` input runs as the B=1 plan and keeps its shape."""
    import torch

    if transform_direction is None:
        transform_direction = "inverse" if transform_type == "c2r" else "forward"
    _validate_semantics(direction, precision, transform_type, transform_direction, norm)
    want = torch.float32 if transform_type == "r2c" else getattr(torch, _SUPPORTED_DTYPES[precision])
    if not isinstance(x, torch.Tensor):
        raise TypeError(f"x must be a torch.Tensor, got {type(x).__name__}")
    if x.dtype != want:
        raise TypeError(f"x must be {want} for transform_type={transform_type} precision={precision}, "
                        f"got {x.dtype}")
    squeezed = False
    if x.dim() == 1:
        n, b = x.numel(), 1
    elif x.dim() == 2 and x.shape[0] == 1:
        x = x[0]
        n, b = x.numel(), 1
        squeezed = True
    elif x.dim() == 2:
        b, n = x.shape
    else:
        raise ValueError(f"x must be rank-1 or rank-2, got dim={x.dim()}")
    if batch is not None and batch != b:
        raise ValueError(f"batch={batch} does not match effective batch {b}")
    if transform_type == "c2r":
        if n < 2:
            raise ValueError(f"c2r half-spectrum length {n} too short")
        n = (n - 1) * 2
    plan = plan_fft(direction, int(n), batch=int(b), precision=precision, profile_hash=profile_hash,
                    table=table, transform_type=transform_type,
                    transform_direction=transform_direction, norm=norm)
    y = execute_fft_plan(plan, x)
    if squeezed:
        y = y.unsqueeze(0)
    return y, plan.as_report()

