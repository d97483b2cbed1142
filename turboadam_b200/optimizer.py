"""TurboAdam on B200: drop-in for the reference optimizer step.

Same constructor, validation, lazy state initialisation, state keys and
bias-correction semantics as reference ``src/turboadam/optimizer.py``. The
per-parameter Python loop of the reference (optimizer.py:88-170, ~20-30
eager launches per CoState tensor) is replaced by one ``ta_step`` call per
device: a fixed sequence of multi-tensor sm_100a kernels over every
parameter of the step.

Stochastic rounding draws come from a counter-based Philox4x32-10 stream
keyed by (seed, tensor id, step, element); the reference draws them from
``torch.rand_like`` / ``rand_buf.uniform_()``, so with the same uniforms the
two produce identical packed state (see tests/).
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch
from torch.optim import Optimizer

from . import _lib
from .costate import CoStateManager
from .oneq import adopt_compressed_v, init_compressed_v, is_padded, storage_capacity

_DTYPES = {torch.float32: _lib.TA_F32, torch.bfloat16: _lib.TA_BF16}


# steps covered by the device bias-correction table of a capturable optimizer
CAPTURE_TABLE_STEPS = 1 << 20


class TurboAdamCommError(RuntimeError):
    """An exchange between the phases of a step whose tensors are split over
    ranks failed (a rank left, a transport error) or ran past its deadline.
    The step stopped part way: parameters and 1Q state are updated, the
    CoState encodings of the split tensors are not, so the optimizer refuses
    further steps until a checkpoint is loaded (``load_state_dict``)."""


# what each exchange of a phased step sums over the ranks
_EXCHANGES = ("alpha chunk sums (after pass 1)", "threshold histogram, round 0",
              "threshold histogram, round 1", "threshold histogram, round 2")


def run_exchanges(gen, process_group=None, timeout=None):
    """Drives a phased step: each region the generator yields is summed over
    the ranks of ``process_group`` in place (all-reduce), then the generator
    resumes; returns what it returns. ``timeout`` (seconds or None): wait on
    the host for each all-reduce with that deadline -- a rank that left or a
    failed transport then ends the step with :class:`TurboAdamCommError`
    instead of a hang; with None the all-reduce is ordered on the current
    stream and only the process group's own timeout bounds it."""
    import datetime

    import torch.distributed as dist

    k = 0
    try:
        region = next(gen)
    except StopIteration as done:
        return done.value
    while True:
        what = _EXCHANGES[k] if k < len(_EXCHANGES) else f"exchange {k}"
        try:
            if timeout is None:
                dist.all_reduce(region, op=dist.ReduceOp.SUM, group=process_group)
            else:
                work = dist.all_reduce(region, op=dist.ReduceOp.SUM, group=process_group,
                                       async_op=True)
                if work.wait(timeout=datetime.timedelta(seconds=float(timeout))) is False:
                    raise RuntimeError(f"no completion within {timeout} s")
        except Exception as e:
            gen.close()
            raise TurboAdamCommError(
                f"exchange {k} of the sharded step ({what}) failed: {e}") from e
        k += 1
        try:
            region = gen.send(None)
        except StopIteration as done:
            return done.value


def _bias_table(betas, steps):
    """fp32 (1 - beta1^t, 1 - beta2^t) for t = 1..steps, each computed in
    Python float arithmetic exactly as the step does (optimizer.py:172-188)."""
    b1, b2 = float(betas[0]), float(betas[1])
    t = np.empty((steps, 2), np.float32)
    t[:, 0] = [1.0 - b1 ** k for k in range(1, steps + 1)]
    t[:, 1] = [1.0 - b2 ** k for k in range(1, steps + 1)]
    return t


class TurboAdam(Optimizer):
    """Adam with CoState-compressed m and 1Q log-scale v (reference API).

    Args mirror the reference (optimizer.py:44-81); ``capturable=True`` (which
    the reference refuses) keeps step counts, bias corrections and the AMP
    loss scale on the device so ``step()`` can be captured into a CUDA graph
    (the first step runs outside capture; gradients must stay at fixed
    addresses). With torch.amp.GradScaler the optimizer takes the
    ``grad_scale`` / ``found_inf`` hand-off (``_step_supports_amp_scaling``):
    gradients are used as ``g * RN(1/scale)``, what ``GradScaler.unscale_``
    would leave, and a step with ``found_inf`` set changes nothing.
    Keyword-only extras:
    ``seed`` keys the stochastic-rounding generator (default
    torch.initial_seed()); ``tensor_ids`` gives each parameter (in the order
    the constructor's param groups list them) the id that keys its rounding
    stream -- by default its position in that order. A rank that steps a
    shard of a larger parameter set passes the shard's global indices
    (``turboadam_b200.sharding.shard_by_tensor``) so its packed state matches
    the unsharded run bit for bit. ``shards`` (same order; None or
    ``(block_offset, global_numel)`` per parameter) marks parameters that are
    slices of a larger tensor split over ranks (ZeRO-1,
    ``turboadam_b200.sharding.zero1_partition``). ``spanning`` lists, in the
    same order on every rank, ``(tensor_id, global_numel)`` of every tensor of
    the job that is split over ranks (``sharding.zero1_spanning``): when it is
    not empty each step runs in phases with the CoState alpha sums and
    threshold histograms all-reduced over ``process_group`` (default group)
    between them -- on every rank, also one that holds no split tensor -- which
    leaves every packed bit equal to the unsharded step's.
    ``exchange_timeout`` (seconds, default None) puts a host deadline on each
    of those all-reduces: a rank that left or a failed collective then ends
    ``step()`` with :class:`TurboAdamCommError` (and the optimizer refuses
    to step again until a checkpoint is loaded) instead of waiting for the
    process group's own timeout.
    ``exact_params=True`` computes the parameter update's v / bc2, square root
    and division correctly rounded, so parameters equal the reference's op
    sequence bit for bit; by default they use the hardware rsqrt / rcp
    estimates (one correction of the quotient): the update is within about
    3e-7 relative of the reference's, inside the 1e-6 parameter tolerance.
    No state depends on the parameters: every packed state bit is the same
    either way.
    """

    # torch.amp.GradScaler hands over `grad_scale` / `found_inf` instead of
    # unscaling the gradients itself
    _step_supports_amp_scaling = True

    def __init__(
        self,
        params,
        lr: float = 1e-3,
        betas: tuple[float, float] = (0.9, 0.999),
        eps: float = 1e-8,
        weight_decay: float = 0.0,
        block_size: int = 128,
        v_bits: int = 4,
        compress_m: bool = True,
        compress_v: bool = True,
        null_pct: float = 0.10,
        amp_pct: float = 0.90,
        error_feedback: bool = False,
        capturable: bool = False,
        min_m_compress_elements: int = 4096,
        *,
        seed: int | None = None,
        tensor_ids=None,
        shards=None,
        spanning=None,
        process_group=None,
        exact_params: bool = False,
        exchange_timeout: float | None = None,
    ):
        if v_bits not in (2, 3, 4, 6, 8):
            raise ValueError(f"v_bits must be one of {{2, 3, 4, 6, 8}}, got {v_bits}")

        defaults = dict(
            lr=lr,
            betas=betas,
            eps=eps,
            weight_decay=weight_decay,
            block_size=block_size,
            v_bits=v_bits,
            compress_m=compress_m,
            compress_v=compress_v,
            null_pct=null_pct,
            amp_pct=amp_pct,
            error_feedback=error_feedback,
            min_m_compress_elements=min_m_compress_elements,
        )
        super().__init__(params, defaults)
        self._group_step_tensors = {}
        self._seed = (torch.initial_seed() if seed is None else int(seed)) & 0xFFFFFFFFFFFFFFFF
        self._tid_override = None
        if tensor_ids is not None:
            flat = [p for g in self.param_groups for p in g["params"]]
            tensor_ids = [int(t) for t in tensor_ids]
            if len(tensor_ids) != len(flat):
                raise ValueError(f"tensor_ids has {len(tensor_ids)} entries for "
                                 f"{len(flat)} parameters")
            if any(t < 0 or t > 0xFFFFFFFF for t in tensor_ids):
                raise ValueError("tensor_ids must be 32-bit unsigned integers")
            self._tid_override = {id(p): t for p, t in zip(flat, tensor_ids)}
        self._shard = {}
        if shards is not None:
            flat = [p for g in self.param_groups for p in g["params"]]
            shards = list(shards)
            if len(shards) != len(flat):
                raise ValueError(f"shards has {len(shards)} entries for {len(flat)} parameters")
            for p, sh in zip(flat, shards):
                if sh is None:
                    continue
                boff, gnumel = int(sh[0]), int(sh[1])
                if boff < 0 or boff * block_size + p.numel() > gnumel:
                    raise ValueError("shard (block_offset, global_numel) does not hold the "
                                     "parameter")
                self._shard[id(p)] = (boff, gnumel)
        self._capturable = bool(capturable)
        self._exact_params = bool(exact_params)
        self._btab = {}
        self._pg = process_group
        self._exchange_timeout = exchange_timeout
        self._failed = None  # why a sharded step stopped part way (TurboAdamCommError)
        self._xbuf = {}
        self._xslot = {}
        self._xbytes = (0, 0)
        if spanning:
            spanning = [(int(t), int(n)) for t, n in spanning]
            gblocks = np.array([-(-n // block_size) for _, n in spanning], dtype=np.int64)
            coff = np.zeros(len(spanning), dtype=np.int64)
            hoff = np.zeros(len(spanning), dtype=np.int64)
            cb, hb = ctypes.c_size_t(0), ctypes.c_size_t(0)
            lib = _lib.load()
            _lib.check(lib.ta_exchange_layout(gblocks.ctypes.data, len(spanning), coff.ctypes.data,
                                              hoff.ctypes.data, ctypes.byref(cb), ctypes.byref(hb)),
                       "ta_exchange_layout")
            self._xslot = {t: (int(c), int(h)) for (t, _), c, h in zip(spanning, coff, hoff)}
            self._xbytes = (cb.value, hb.value)
        self._plans = None
        self._ready = set()  # id() of parameters whose state is fully initialised
        self._devices = set()  # devices of those parameters
        self._bc_cache = {}  # (beta1, beta2, step) -> fp32 bias corrections
        self._ws = {}
        # test hook: {"uniforms": {param: fp32 [B*128] cuda}, "alpha": {param: fp32 [1] cuda}}
        self._parity = None
        # timing hook: 5 recorded torch.cuda.Event objects marking the kernel
        # phases of the next step(s) (see ta_step_profiled)
        self._phase_events = None

    # ------------------------------------------------------------------
    # state dict
    # ------------------------------------------------------------------
    def add_param_group(self, param_group):
        super().add_param_group(param_group)
        self._plans = None
        if hasattr(self, "_ready"):
            self._ready.clear()
            self._devices.clear()

    def load_state_dict(self, state_dict):
        """Load and re-home packed state into the padded device layout
        (reference optimizer.py:194-218 migrates CoState tensors by hand).

        Takes this optimizer's own state dicts and the reference's: a
        ``m_mgr`` of another class with the reference CoStateManager's
        attributes (the reference's class itself, or the stand-in that
        ``turboadam_b200.checkpoint.load_reference_state_dict`` unpickles it
        as) is converted to this package's manager; 1Q headers that torch
        cast to the parameter dtype go back to fp16 (exact); the reference's
        CUDA ``rand_buf`` is dropped (the draws are Philox here)."""
        super().load_state_dict(state_dict)
        self._failed = None
        self._ready.clear()
        self._devices.clear()
        for group in self.param_groups:
            for p in group["params"]:
                if p not in self.state:
                    continue
                st = self.state[p]
                if "compressed_v" in st and not is_padded(st["compressed_v"], p.device):
                    st["compressed_v"] = adopt_compressed_v(st["compressed_v"], p.device)
                mgr = st.get("m_mgr")
                if mgr is not None and not isinstance(mgr, CoStateManager):
                    mgr = CoStateManager.from_reference(mgr)
                    st["m_mgr"] = mgr
                if isinstance(mgr, CoStateManager):
                    mgr.adopt(p.numel(), p.device, p.shape)
                for k in ("exp_avg", "exp_avg_sq"):
                    if k in st:
                        st[k] = st[k].to(device=p.device, dtype=torch.float32).contiguous()
                for k in ("_bc1", "_bc2"):
                    if k in st:
                        st[k] = st[k].to(device=p.device, dtype=torch.float32)
        self._plans = None

    # ------------------------------------------------------------------
    # step
    # ------------------------------------------------------------------
    def _init_state(self, group_idx, group, p):
        state = self.state[p]
        block_size = group["block_size"]
        if len(state) == 0:  # optimizer.py:243-269
            state["step"] = 0
            # the policy looks at the whole tensor, so every rank of a split
            # tensor makes the same choice
            gnumel = self._shard.get(id(p), (0, p.numel()))[1]
            compress_this_m = group["compress_m"] and gnumel >= group["min_m_compress_elements"]
            state["_compress_m"] = compress_this_m
            if compress_this_m:
                mgr = CoStateManager(block_size=block_size, null_pct=group["null_pct"],
                                     amp_pct=group["amp_pct"],
                                     error_feedback=group["error_feedback"])
                mgr.allocate(p.numel(), p.device, p.shape)
                state["m_mgr"] = mgr
            else:
                state["exp_avg"] = torch.zeros_like(p, dtype=torch.float32,
                                                    memory_format=torch.contiguous_format)
            if not group["compress_v"]:
                state["exp_avg_sq"] = torch.zeros_like(p, dtype=torch.float32,
                                                       memory_format=torch.contiguous_format)
            key = (group_idx, p.device.type, p.device.index)
            if key not in self._group_step_tensors:
                self._group_step_tensors[key] = {
                    "bc1": torch.empty(1, dtype=torch.float32, device=p.device),
                    "bc2": torch.empty(1, dtype=torch.float32, device=p.device),
                }
            gt = self._group_step_tensors[key]
            state["_bc1"] = gt["bc1"]
            state["_bc2"] = gt["bc2"]
            self._plans = None
        if group["compress_v"] and "compressed_v" not in state:  # optimizer.py:273-280
            state["compressed_v"] = init_compressed_v(p.shape, group["v_bits"], p.device,
                                                      block_size)
            self._plans = None

    def _bias_corrections(self):
        """optimizer.py:172-188: per group, the last param holding state wins
        (found from the end of the group; the fp32 values are cached per
        (betas, step))."""
        out = {}
        ready = self._ready
        for gi, group in enumerate(self.param_groups):
            beta1, beta2 = group["betas"]
            for p in reversed(group["params"]):
                if id(p) not in ready and p not in self.state:
                    continue
                nxt = self.state[p]["step"] + 1
                key = (beta1, beta2, nxt)
                bc = self._bc_cache.get(key)
                if bc is None:
                    if len(self._bc_cache) > 4096:
                        self._bc_cache.clear()
                    bc = (np.float32(1.0 - beta1 ** nxt), np.float32(1.0 - beta2 ** nxt))
                    self._bc_cache[key] = bc
                out[gi] = bc
                break
        return out

    @torch.no_grad()
    def step(self, closure=None):
        """Perform a single optimization step."""
        if self._failed is not None:
            raise TurboAdamCommError(
                f"a previous step stopped part way ({self._failed}); load a checkpoint "
                "(load_state_dict) before stepping again")
        try:
            return run_exchanges(self._step_gen(closure), self._pg, self._exchange_timeout)
        except TurboAdamCommError as e:
            self._failed = str(e)
            raise

    def _step_gen(self, closure=None):
        """The step as a generator: yields each exchange region (fp64 alpha
        chunk sums, then int32 histograms) that must be summed over the ranks
        in place before it is resumed; returns the closure's loss."""
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()

        work = []
        ready = self._ready
        for gi, group in enumerate(self.param_groups):
            for p in group["params"]:
                if p.grad is None:
                    continue
                if id(p) not in ready:  # checks and lazy state, once per parameter
                    _lib.require_cuda(p)
                    if p.dtype not in _DTYPES:
                        raise NotImplementedError(
                            f"param dtype {p.dtype}: the sm_100a step is built for float32 and "
                            "bfloat16 parameters")
                    if group["block_size"] != 128:
                        raise NotImplementedError(
                            "block_size != 128 is not built for the device step")
                    self._init_state(gi, group, p)
                    ready.add(id(p))
                    self._devices.add(p.device)
                work.append((gi, p))
        if not work:
            return loss
        gs = getattr(self, "grad_scale", None)
        fi = getattr(self, "found_inf", None)
        if self._capturable:
            by_dev = {}
            for gi, p in work:
                by_dev.setdefault(p.device, []).append((gi, p))
            for dev, items in by_dev.items():
                self._run_device_capturable(dev, items, gs, fi)
            return loss
        if fi is not None and float(fi) != 0.0:
            return loss  # GradScaler skips a step whose gradients overflowed
        if gs is not None:  # GradScaler.unscale_: g *= RN(1 / scale), in place
            inv = gs.double().reciprocal().float()
            dummy = torch.zeros(1, dtype=torch.float32, device=inv.device)
            for dev in {p.device for _, p in work}:
                grads = [p.grad for _, p in work if p.device == dev]
                f32 = [g for g in grads if g.dtype == torch.float32]
                if f32:
                    torch._amp_foreach_non_finite_check_and_unscale_(f32, dummy.to(dev),
                                                                     inv.to(dev))
                for g in grads:  # bf16: the fp32 product rounded back (as on the device)
                    if g.dtype != torch.float32:
                        g.mul_(inv.to(dev))
        bcs = self._bias_corrections()
        for gi, (bc1, bc2) in bcs.items():
            for key, gt in self._group_step_tensors.items():
                if key[0] == gi:
                    gt["bc1"].fill_(float(bc1))
                    gt["bc2"].fill_(float(bc2))

        if len(self._devices) == 1:
            by_dev = {next(iter(self._devices)): work}
        else:
            by_dev = {}
            for gi, p in work:
                by_dev.setdefault(p.device, []).append((gi, p))
        for dev, items in by_dev.items():
            yield from self._run_device(dev, items, bcs)
        return loss

    # ------------------------------------------------------------------
    def _tensor_ids(self):
        ids = {}
        i = 0
        over = self._tid_override or {}
        for group in self.param_groups:
            for p in group["params"]:
                ids.setdefault(id(p), over.get(id(p), i))
                i += 1
        return ids

    def _build_plan(self, dev, items):
        lib = _lib.load()
        tids = self._tensor_ids()
        n = len(items)
        arr = np.zeros(n, dtype=_lib.TENSOR_DTYPE)
        for i, (gi, p) in enumerate(items):
            st = self.state[p]
            group = self.param_groups[gi]
            r = arr[i]
            r["param_dev"] = p.data_ptr()
            r["numel"] = p.numel()
            r["dtype"] = _DTYPES[p.dtype]
            r["group"] = gi
            r["tensor_id"] = tids[id(p)] & 0xFFFFFFFF
            flags = _lib.TA_EXACT_PARAM if self._exact_params else 0
            sh = self._shard.get(id(p))
            if sh is not None:
                boff, gnumel = sh
                gblocks = -(-gnumel // group["block_size"])
                r["block_offset"] = boff
                r["global_blocks"] = gblocks
                if st["_compress_m"] and (boff != 0 or -(-p.numel() // group["block_size"]) != gblocks):
                    flags |= _lib.TA_M_SPANNING
                    slot = self._xslot.get(tids[id(p)])
                    if slot is None:
                        raise ValueError(f"tensor {tids[id(p)]} is split over ranks but missing "
                                         "from `spanning`")
                    r["exch_chunk_off"], r["exch_hist_off"] = slot
            if st["_compress_m"]:
                mgr = st["m_mgr"]
                flags |= _lib.TA_M_COSTATE
                lab, sgn, nrm, amp, alpha = mgr.pointers()
                r["m_labels_dev"], r["m_signs_dev"], r["m_norms_dev"] = lab, sgn, nrm
                r["m_amp_dev"], r["m_alpha_dev"] = amp, alpha
                if mgr._error_feedback:
                    flags |= _lib.TA_M_EF
                    r["m_ef_dev"] = mgr.ef_pointer()
            else:
                r["exp_avg_dev"] = st["exp_avg"].data_ptr()
            if group["compress_v"]:
                flags |= _lib.TA_V_ONEQ
                cv = st["compressed_v"]
                r["v_idx_dev"] = cv["indices"].data_ptr()
                r["v_hdr_dev"] = cv["scales"].data_ptr()
            else:
                r["exp_avg_sq_dev"] = st["exp_avg_sq"].data_ptr()
            r["flags"] = flags
            if p.data_ptr() % 16 != 0:
                raise NotImplementedError("parameter storage must be 16-byte aligned")
        ws_bytes = lib.ta_workspace_size(arr.ctypes.data, n)
        ws = self._ws.get(dev)
        if ws is None or ws.numel() < ws_bytes:
            ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
            self._ws[dev] = ws
        groups = np.zeros(len(self.param_groups), dtype=_lib.GROUP_DTYPE)
        cb, hb = self._xbytes
        if cb + hb:
            if len({pp.device for _, pp in items}) != 1 or (self._xbuf and dev not in self._xbuf):
                raise NotImplementedError("a sharded step keeps all of a rank's parameters on one "
                                          "device")
            xb = self._xbuf.get(dev)
            if xb is None:
                xb = torch.zeros(cb + hb, dtype=torch.uint8, device=dev)
                self._xbuf[dev] = xb
        ps = [p for _, p in items]
        sts = [self.state[p] for p in ps]
        return {"key": tuple(id(p) for p in ps), "arr": arr, "groups": groups,
                "xbytes": cb + hb, "chunk_bytes": cb, "hist_bytes": hb,
                # per-step fast path: the parameters, their state dicts and
                # managers in plan order, the parameter storage the table
                # points at, and whether every manager already holds state
                "params": ps, "states": sts, "mgrs": [st.get("m_mgr") for st in sts],
                "pdtypes": [p.dtype for p in ps], "pptrs": [p.data_ptr() for p in ps],
                "settled": False, "parity_set": False}

    def _refresh_grads(self, plan):
        """Points the plan's table at this step's gradients; returns the
        tensors to keep alive until the step is enqueued. The common case --
        contiguous, 16-byte aligned gradients of the parameter's dtype -- is
        one pass over the list."""
        ps = plan["params"]
        grads = [p.grad for p in ps]
        gptrs = [g.data_ptr() for g in grads]
        if ([g.dtype for g in grads] == plan["pdtypes"]
                and all([g.is_contiguous() for g in grads]) and not any([x & 15 for x in gptrs])):
            plan["arr"]["grad_dev"] = gptrs
            return grads
        keep = []
        grad_ptr = plan["arr"]["grad_dev"]
        for i, (p, g) in enumerate(zip(ps, grads)):
            if g.dtype != p.dtype:
                if p.dtype == torch.float32 and g.dtype == torch.bfloat16:
                    g = g.float()
                else:
                    raise NotImplementedError(f"grad dtype {g.dtype} with param dtype {p.dtype}")
            if not g.is_contiguous() or g.data_ptr() % 16:
                g = g.contiguous().clone() if g.data_ptr() % 16 else g.contiguous()
            keep.append(g)
            grad_ptr[i] = g.data_ptr()
        return keep

    def _run_device(self, dev, items, bcs):
        lib = _lib.load()
        if self._plans is None:
            self._plans = {}
        plan = self._plans.get(dev)
        key = tuple([id(p) for _, p in items])
        if (plan is None or plan["key"] != key
                or [p.data_ptr() for p in plan["params"]] != plan["pptrs"]):
            plan = self._build_plan(dev, items)
            self._plans[dev] = plan
        arr = plan["arr"]
        keep = self._refresh_grads(plan)
        sts = plan["states"]
        for st in sts:
            st["step"] += 1  # optimizer.py:103
        arr["step"] = [st["step"] for st in sts]
        settled = plan["settled"]
        if not settled:
            # the CoState flags change until every manager holds an encoding
            # (and, with error feedback, a residual); then they stay put
            flags = arr["flags"]
            settled = True
            for i, mgr in enumerate(plan["mgrs"]):
                if mgr is None:
                    continue
                f = int(flags[i]) & ~(_lib.TA_M_HAS_STATE | _lib.TA_M_EF_STATE)
                if mgr._has_state:
                    f |= _lib.TA_M_HAS_STATE
                if mgr._ef_residual is not None:
                    f |= _lib.TA_M_EF_STATE
                flags[i] = f
                settled = settled and mgr._has_state and (
                    not mgr._error_feedback or mgr._ef_residual is not None)
        parity = self._parity
        if parity is not None or plan["parity_set"]:
            uni = arr["sr_uniforms_dev"]
            ainj = arr["alpha_inject_dev"]
            plan["parity_set"] = parity is not None
            for i, p in enumerate(plan["params"]):
                if parity is not None:
                    u = parity.get("uniforms", {}).get(p)
                    a = parity.get("alpha", {}).get(p)
                    uni[i] = u.data_ptr() if u is not None else 0
                    ainj[i] = a.data_ptr() if a is not None else 0
                    keep += [u, a]
                else:
                    uni[i] = 0
                    ainj[i] = 0
        groups = plan["groups"]
        self._fill_groups(groups, bcs)
        ws = self._ws[dev]
        if plan["xbytes"]:  # tensors split over ranks: the phased step
            xb = self._xbuf[dev]
            cb, hb = plan["chunk_bytes"], plan["hist_bytes"]
            evs = self._phase_events
            cur = torch.cuda.current_stream(dev)
            for phase in range(_lib.TA_PHASE_LABELS + 1):
                if evs is not None and phase == _lib.TA_PHASE_PASS1:
                    evs[0].record(cur)
                with torch.cuda.device(dev):
                    rc = lib.ta_step_phase(arr.ctypes.data, len(items), groups.ctypes.data,
                                           len(groups), self._seed, ws.data_ptr(), ws.numel(),
                                           xb.data_ptr(), cb, hb, phase, _lib.stream_ptr(dev))
                _lib.check(rc, "ta_step_phase")
                if evs is not None:  # pass 1 | (alpha) | alpha, pass 2 | select, labels
                    if phase == _lib.TA_PHASE_PASS1:
                        evs[1].record(cur)
                        evs[2].record(cur)
                    elif phase == _lib.TA_PHASE_PASS2:
                        evs[3].record(cur)
                    elif phase == _lib.TA_PHASE_LABELS:
                        evs[4].record(cur)
                if phase == _lib.TA_PHASE_PASS1:
                    yield xb[:cb].view(torch.float64)
                elif phase < _lib.TA_PHASE_LABELS:
                    yield xb[cb:cb + hb].view(torch.int32)
            self._mark_updated(plan, settled)
            del keep
            return
        with torch.cuda.device(dev):
            if self._phase_events is None:
                rc = lib.ta_step(arr.ctypes.data, len(items), groups.ctypes.data, len(groups),
                                 self._seed, ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
            else:
                evs = (ctypes.c_void_p * 5)(*[e.cuda_event for e in self._phase_events])
                rc = lib.ta_step_profiled(arr.ctypes.data, len(items), groups.ctypes.data,
                                          len(groups), self._seed, ws.data_ptr(), ws.numel(),
                                          _lib.stream_ptr(dev), evs)
        _lib.check(rc, "ta_step")
        self._mark_updated(plan, settled)
        # Temporaries in `keep` were allocated on the current stream, so the
        # caching allocator only reuses them for work ordered after ta_step.
        del keep

    @staticmethod
    def _mark_updated(plan, settled):
        """Exposes the managers' new encodings (nothing to do once every
        manager of the plan held state before this step)."""
        if settled:
            plan["settled"] = True
            return
        for mgr in plan["mgrs"]:
            if mgr is not None:
                mgr.mark_updated()

    def _fill_groups(self, groups, bcs):
        for gi, group in enumerate(self.param_groups):
            g = groups[gi]
            lr = group["lr"]
            g["lr"] = float(lr) if not isinstance(lr, torch.Tensor) else float(lr.item())
            g["beta1"], g["beta2"] = group["betas"]
            g["eps"] = group["eps"]
            g["weight_decay"] = group["weight_decay"]
            g["null_pct"] = group["null_pct"]
            g["amp_pct"] = group["amp_pct"]
            bc = bcs.get(gi, (np.float32(1.0), np.float32(1.0)))
            g["bc1"], g["bc2"] = bc
            g["block_size"] = group["block_size"]
            g["v_bits"] = group["v_bits"]

    # ------------------------------------------------------------------
    def _run_device_capturable(self, dev, items, gs, fi):
        """capturable=True: the plan (descriptor table, step counts, bias
        table) is uploaded once; each step is ta_step_prepared, kernel
        launches only."""
        lib = _lib.load()
        if self._plans is None:
            self._plans = {}
        plan = self._plans.get(dev)
        key = tuple(id(p) for _, p in items)
        gptrs = tuple(p.grad.data_ptr() for _, p in items)
        if plan is None or plan["key"] != key or plan.get("gptrs") != gptrs:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("the first capturable step, and any change of parameters or "
                                   "gradient storage, must run outside CUDA graph capture")
            for _, p in items:
                g = p.grad
                if g.dtype != p.dtype or not g.is_contiguous() or g.data_ptr() % 16:
                    raise NotImplementedError("capturable steps need contiguous, 16-byte aligned "
                                              "gradients of the parameter's dtype")
            plan = self._build_plan(dev, items)
            arr = plan["arr"]
            steps = []
            for i, (gi, p) in enumerate(items):
                st = self.state[p]
                s0 = st["step"]
                s0 = int(s0.item()) if isinstance(s0, torch.Tensor) else int(s0)
                steps.append(s0)
                arr[i]["grad_dev"] = p.grad.data_ptr()
                arr[i]["step"] = s0 + 1
                mgr = st.get("m_mgr")
                if mgr is not None and mgr._has_state:
                    arr[i]["flags"] = int(arr[i]["flags"]) | _lib.TA_M_HAS_STATE
            groups = plan["groups"]
            self._fill_groups(groups, {})
            tables = []
            for g in self.param_groups:
                k = (float(g["betas"][0]), float(g["betas"][1]))
                if k not in self._btab:
                    self._btab[k] = _bias_table(k, CAPTURE_TABLE_STEPS)
                tables.append(self._btab[k])
            plan["table"] = torch.from_numpy(np.stack(tables)).to(dev)
            plan["steps"] = torch.tensor(steps, dtype=torch.int32, device=dev)
            plan["gptrs"] = gptrs
            with torch.cuda.device(dev):
                rc = lib.ta_plan_prepare(arr.ctypes.data, len(items), groups.ctypes.data,
                                         len(groups), self._seed, self._ws[dev].data_ptr(),
                                         self._ws[dev].numel(), _lib.stream_ptr(dev))
            _lib.check(rc, "ta_plan_prepare")
            for i, (gi, p) in enumerate(items):
                self.state[p]["step"] = plan["steps"][i]
            self._plans[dev] = plan
        lr_ptr = None
        if any(isinstance(g["lr"], torch.Tensor) for g in self.param_groups):
            if "lr" not in plan:
                plan["lr"] = torch.zeros(len(self.param_groups), dtype=torch.float64, device=dev)
            for gi, g in enumerate(self.param_groups):
                if isinstance(g["lr"], torch.Tensor):
                    plan["lr"][gi].copy_(g["lr"])
                else:
                    plan["lr"][gi].fill_(float(g["lr"]))
            lr_ptr = plan["lr"].data_ptr()
        for t in (gs, fi):
            if t is not None and (t.device != dev or t.dtype != torch.float32):
                raise NotImplementedError("grad_scale / found_inf must be float32 tensors on "
                                          "the parameters' device")
        dyn = _lib.TaDynamic(plan["steps"].data_ptr(), plan["table"].data_ptr(),
                             CAPTURE_TABLE_STEPS, lr_ptr,
                             gs.data_ptr() if gs is not None else None,
                             fi.data_ptr() if fi is not None else None)
        ws = self._ws[dev]
        with torch.cuda.device(dev):
            rc = lib.ta_step_prepared(plan["arr"].ctypes.data, len(items),
                                      plan["groups"].ctypes.data, len(plan["groups"]),
                                      self._seed, ws.data_ptr(), ws.numel(), ctypes.byref(dyn),
                                      _lib.stream_ptr(dev))
        _lib.check(rc, "ta_step_prepared")
        for _, p in items:
            mgr = self.state[p].get("m_mgr")
            if mgr is not None:
                mgr.mark_updated()

    # ------------------------------------------------------------------
    def read_status(self, clear: bool = True) -> int:
        """Device status bits accumulated since the last read
        (TA_STATUS_NONFINITE_GRAD, TA_STATUS_WAIT_TIMEOUT)."""
        lib = _lib.load()
        out = 0
        for dev, ws in self._ws.items():
            v = ctypes.c_uint32(0)
            _lib.check(lib.ta_read_status(ws.data_ptr(), int(clear), ctypes.byref(v),
                                          _lib.stream_ptr(dev)), "ta_read_status")
            out |= v.value
        return out


def _single_costate_update(mgr: CoStateManager, g: torch.Tensor, beta1: float,
                           uniforms=None, alpha_inject=None) -> torch.Tensor:
    """CoStateManager.update (costate.py:367-464) through ta_step with
    TA_NO_PARAM: decode, EMA, alpha, encode, thresholds, labels."""
    _lib.require_cuda(g)
    lib = _lib.load()
    dev = g.device
    gf = g.reshape(-1)
    if gf.dtype not in (torch.float32, torch.bfloat16):
        gf = gf.float()
    gf = gf.contiguous()
    n = gf.numel()
    if mgr._bufs is None:
        mgr.allocate(n, dev, g.shape)
    arr = np.zeros(1, dtype=_lib.TENSOR_DTYPE)
    r = arr[0]
    r["grad_dev"] = gf.data_ptr()
    r["numel"] = n
    r["dtype"] = _DTYPES[gf.dtype]
    r["flags"] = _lib.TA_M_COSTATE | _lib.TA_NO_PARAM | (
        _lib.TA_M_HAS_STATE if mgr._has_state else 0)
    if mgr._error_feedback:
        r["flags"] |= _lib.TA_M_EF | (_lib.TA_M_EF_STATE if mgr._ef_residual is not None else 0)
        r["m_ef_dev"] = mgr.ef_pointer()
    r["step"] = 1
    lab, sgn, nrm, amp, alpha = mgr.pointers()
    r["m_labels_dev"], r["m_signs_dev"], r["m_norms_dev"] = lab, sgn, nrm
    r["m_amp_dev"], r["m_alpha_dev"] = amp, alpha
    m_out = torch.empty(n, dtype=torch.float32, device=dev)
    r["m_out_dev"] = m_out.data_ptr()
    if alpha_inject is not None:
        r["alpha_inject_dev"] = alpha_inject.data_ptr()
    groups = np.zeros(1, dtype=_lib.GROUP_DTYPE)
    gr = groups[0]
    gr["beta1"] = beta1
    gr["beta2"] = 0.999
    gr["null_pct"] = mgr._null_pct
    gr["amp_pct"] = mgr._amp_pct
    gr["bc1"] = gr["bc2"] = 1.0
    gr["block_size"] = mgr.block_size
    gr["v_bits"] = 4
    ws = torch.zeros(lib.ta_workspace_size(arr.ctypes.data, 1), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.check(lib.ta_step(arr.ctypes.data, 1, groups.ctypes.data, 1, 0, ws.data_ptr(),
                               ws.numel(), _lib.stream_ptr(dev)), "ta_step")
    mgr.mark_updated()
    return m_out.reshape(g.shape)
