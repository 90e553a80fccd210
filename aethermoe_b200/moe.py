"""The composed MoE layer on B200: single-GPU (``MoELayer``) and expert-parallel
over NCCL (``EPLayer``), thin Python owners of the C-ABI handles.

Device buffers are torch CUDA tensors (plumbing only); every kernel is in
``libaethermoe.so``.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib

_vp = ctypes.c_void_p


def _dtype_code(t):
    import torch
    if t.dtype == torch.float32:
        return _lib.F32
    if t.dtype == torch.bfloat16:
        return _lib.BF16
    raise ValueError(f"unsupported dtype {t.dtype} (float32 or bfloat16)")


def _stream_ptr(stream):
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


def make_config(d_model, d_ffn, num_experts, top_k, capacity=None, gating_mode=_lib.GATING_EXACT):
    cfg = _lib.MoeConfig()
    cfg.d_model = d_model
    cfg.d_ffn = d_ffn
    cfg.num_experts = num_experts
    cfg.top_k = top_k
    cfg.capacity = _lib.CAPACITY_UNLIMITED if capacity is None else int(capacity)
    cfg.gating_mode = gating_mode
    return cfg


class MoELayer:
    """gating -> capacity routing -> grouped INT8 expert FFN (up, ReLU, down) -> combine.

    ``gate_w [d, E]``, ``gate_b [E]``; ``q_up [E, d, ffn]`` int8 with
    ``s_up [E, ffn]``; ``q_down [E, ffn, d]`` with ``s_down [E, d]`` (the
    reference's per-output-column quantisation layout, one group per expert).
    """

    def __init__(self, gate_w, gate_b, q_up, s_up, q_down, s_down, top_k, capacity=None,
                 gating_mode=_lib.GATING_EXACT, device=0):
        gate_w = np.asarray(gate_w, np.float32)
        d, e = gate_w.shape
        self.device = device
        self.gate = _lib.Gate(gate_w, gate_b, device)
        if isinstance(q_up, _lib.QWeight):  # already packed (e.g. DeviceQWeight)
            self.up, self.down = q_up, q_down
            ffn = q_up.N
        else:
            ffn = np.shape(q_up)[2]
            self.up = _lib.QWeight(q_up, np.asarray(s_up, np.float32).reshape(e, ffn), device)
            self.down = _lib.QWeight(q_down, np.asarray(s_down, np.float32).reshape(e, d), device)
        self.cfg = make_config(d, ffn, e, top_k, capacity, gating_mode)
        h = _vp()
        _lib.check(_lib.lib().aem_moe_create(ctypes.byref(self.cfg), self.gate.handle,
                                             self.up.handle, self.down.handle, ctypes.byref(h)),
                   "aem_moe_create")
        self.handle = h.value
        self.d_model, self.d_ffn, self.num_experts, self.top_k = d, ffn, e, top_k

    def forward(self, x, out=None, out_dtype=None, stream=None):
        """``x`` torch CUDA tensor [T, d] (float32/bfloat16) -> [T, d]."""
        import torch
        t = x.shape[0]
        if out is None:
            out = torch.empty((t, self.d_model), dtype=out_dtype or x.dtype, device=x.device)
        _lib.check(_lib.lib().aem_moe_forward(self.handle, x.data_ptr(), _dtype_code(x), t,
                                              out.data_ptr(), _dtype_code(out), _stream_ptr(stream)),
                   "aem_moe_forward")
        return out

    def forward_slices(self, slices, out_dtype=None, stream=None):
        """One scheduler iteration as one batch: ``slices`` is a list of
        ``(seq_id, x)`` with ``x`` a CUDA tensor [tokens, d] (decode steps and
        prefill chunks, in the scheduler's order).  Returns the output tensors
        in the same order (``aem_moe_forward_slices``)."""
        import torch
        if not slices:
            return []
        xd = slices[0][1]
        outs = [torch.empty((x.shape[0], self.d_model), dtype=out_dtype or xd.dtype,
                            device=x.device) for _, x in slices]
        arr = (_lib.SeqSlice * len(slices))()
        for i, ((sid, x), o) in enumerate(zip(slices, outs)):
            if x.dtype != xd.dtype:
                raise ValueError("all slices must share one dtype")
            arr[i] = _lib.SeqSlice(int(sid), x.data_ptr(), o.data_ptr(), int(x.shape[0]))
        _lib.check(_lib.lib().aem_moe_forward_slices(self.handle, arr, len(slices),
                                                     _dtype_code(xd), _dtype_code(outs[0]),
                                                     _stream_ptr(stream)),
                   "aem_moe_forward_slices")
        return outs

    def forward_host(self, x, out_dtype=np.float32):
        """Host buffers through ``aem_moe_forward_host`` (copies included)."""
        x = np.ascontiguousarray(x)
        if x.dtype == np.float32:
            xd = _lib.F32
        elif x.dtype == np.uint16:  # raw bfloat16 bits
            xd = _lib.BF16
        else:
            raise ValueError("x must be float32 or raw bfloat16 (uint16)")
        od = _lib.F32 if np.dtype(out_dtype) == np.float32 else _lib.BF16
        out = np.empty((x.shape[0], self.d_model), dtype=np.float32 if od == _lib.F32 else np.uint16)
        _lib.check(_lib.lib().aem_moe_forward_host(_lib.context(self.device), self.handle,
                                                   x.ctypes.data, xd, x.shape[0], out.ctypes.data,
                                                   od), "aem_moe_forward_host")
        return out

    def set_hidden_dtype(self, dtype):
        """Storage of the hidden activation: ``None`` (follow x), ``"f32"``
        (a bf16 hi + lo pair) or ``"bf16"`` (``aem_moe_set_hidden_dtype``)."""
        code = {None: -1, "f32": _lib.F32, "bf16": _lib.BF16}[dtype]
        _lib.check(_lib.lib().aem_moe_set_hidden_dtype(self.handle, code), "aem_moe_set_hidden_dtype")

    def profile(self, enable=True):
        _lib.check(_lib.lib().aem_moe_profile(self.handle, 1 if enable else 0), "aem_moe_profile")

    def profile_read(self):
        """``({phase: summed ms}, steps)`` since profiling was enabled."""
        ms = (ctypes.c_double * _lib.NUM_PHASES)()
        steps = ctypes.c_int64()
        _lib.check(_lib.lib().aem_moe_profile_read(self.handle, ms, ctypes.byref(steps)))
        return dict(zip(_lib.PHASES, list(ms))), steps.value

    def last_routing(self, T, stream=None):
        """``(idx [T, k(+1)], val [T, k], effective [T*k])`` of the last forward, as torch tensors."""
        import torch
        k, e = self.top_k, self.num_experts
        ksel = k + 1 if k < e else k
        dev = torch.device("cuda", self.device)
        idx = torch.empty((T, ksel), dtype=torch.int32, device=dev)
        val = torch.empty((T, k), dtype=torch.float32, device=dev)
        eff = torch.empty((T * k,), dtype=torch.int32, device=dev)
        _lib.check(_lib.lib().aem_moe_last_routing(self.handle, idx.data_ptr(), val.data_ptr(),
                                                   eff.data_ptr(), _stream_ptr(stream)),
                   "aem_moe_last_routing")
        return idx, val, eff

    def close(self):
        if getattr(self, "handle", None):
            _lib.lib().aem_moe_free(self.handle)
            self.handle = None
        for w in ("gate", "up", "down"):
            if getattr(self, w, None) is not None:
                getattr(self, w).close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ep_unique_id():
    buf = (ctypes.c_uint8 * 128)()
    _lib.check(_lib.lib().aem_ep_unique_id(buf), "aem_ep_unique_id")
    return bytes(buf)


def ep_plan_bases(counts, rank):
    """Host planning of the distributed capacity rule: ``counts [R, k, E]`` -> ``base [k, E]``."""
    c = np.ascontiguousarray(counts, dtype=np.int64)
    r, k, e = c.shape
    base = np.zeros((k, e), dtype=np.int64)
    _lib.check(_lib.lib().aem_ep_plan_bases(c.ctypes.data, r, k, e, rank, base.ctypes.data),
               "aem_ep_plan_bases")
    return base


def ep_plan_exchange(starts, rank):
    """Host planning of one exchange: ``starts [R, E+1]`` (every rank's expert
    starts) -> ``(send_off, send_cnt, recv_off, recv_cnt, groups)`` for ``rank``."""
    st = np.ascontiguousarray(starts, dtype=np.int32)
    r, e1 = st.shape
    e = e1 - 1
    so, sc, ro, rc = (np.zeros(r, np.int64) for _ in range(4))
    groups = np.zeros(e + 1, np.int32)
    _lib.check(_lib.lib().aem_ep_plan_exchange(st.ctypes.data, r, e, rank, so.ctypes.data,
                                               sc.ctypes.data, ro.ctypes.data, rc.ctypes.data,
                                               groups.ctypes.data), "aem_ep_plan_exchange")
    return so, sc, ro, rc, groups


def ep_payload(eff, T, E, R, live=None):
    """One rank's exchange payload from its routing (``eff`` slot-major
    ``[k*T]`` expert positions, experts in contiguous blocks of E/R per rank):
    expert starts, pair counts per destination, live mask, half-A units per
    expert, half-A pairs per destination (half A = the first ceil(T/2))."""
    eff = np.asarray(eff).reshape(-1, T)
    el, half = E // R, (T + 1) // 2
    if live is None:
        live = (1 << R) - 1
    row = np.zeros(_lib.ep_payload_words(E, R), np.int32)
    row[1:E + 1] = np.cumsum(np.bincount(eff.reshape(-1), minlength=E))
    dest = eff // el
    for r in range(R):
        if (live >> r) & 1:
            on = (dest == r).any(axis=0)
            row[E + 1 + r] = on.sum()
            row[2 * E + 3 + R + r] = on[:half].sum()
    row[E + 1 + R:E + 3 + R] = np.array([live & 0xFFFFFFFF, (live >> 32) & 0xFFFFFFFF],
                                        np.uint32).view(np.int32)
    row[E + 3 + R:2 * E + 3 + R] = np.bincount(eff[:, :half].reshape(-1), minlength=E)
    return row


def ep_plan_peer(payload, rank, units_cap, pairs_cap, ret_cap, live=None):
    """Host form of the per-step peer-exchange plan: ``payload [R, W]``
    (every rank's ``ep_payload``) -> ``(plan dict, groups [2, E/R+1])`` for
    ``rank`` (received rows per local expert, per half); ``live`` is the bit
    mask of the ranks taking part (default: all)."""
    pay = np.ascontiguousarray(payload, dtype=np.int32)
    r = pay.shape[0]
    e = None
    for cand in range(1, 257):  # E from the row width
        if _lib.ep_payload_words(cand, r) == pay.shape[1] and cand % r == 0:
            e = cand
    if e is None:
        raise ValueError(f"payload width {pay.shape[1]} fits no expert count for {r} ranks")
    if live is None:
        live = (1 << r) - 1
    plan = _lib.EpPeerPlan()
    groups = np.zeros(2 * (e + 1), np.int32)
    _lib.check(_lib.lib().aem_ep_plan_peer(pay.ctypes.data, r, e, rank, int(live), units_cap,
                                           pairs_cap, ret_cap, ctypes.byref(plan),
                                           groups.ctypes.data), "aem_ep_plan_peer")
    el = e // r
    out = dict(ok=plan.ok, units_in=plan.units_in, units_in_a=plan.units_in_a,
               pairs_in=plan.pairs_in, pairs_out=plan.pairs_out)
    for name in ("dst_pair_off", "send_pair_off", "send_pair_a", "recv_pair_a", "ret_off"):
        out[name] = np.array(getattr(plan, name)[:r], np.int64)
    out["dst_unit_off"] = np.array([list(plan.dst_unit_off[h])[:e] for h in range(2)], np.int64)
    out["recv_pair_off"] = np.array(plan.recv_pair_off[:r + 1], np.int64)
    return out, groups[:2 * (el + 1)].reshape(2, el + 1)


class EPLayer:
    """One rank of the expert-parallel MoE layer (experts split contiguously over ranks).

    Collective: every rank constructs it with the same config, placement and
    ``max_tokens`` (the most tokens one rank passes to one ``forward``).
    ``expert_to_rank`` [E] places the experts (None = contiguous blocks); the
    local weights hold this rank's experts in increasing expert id."""

    def __init__(self, uid, rank, world, gate_w, gate_b, q_up_local, s_up_local, q_down_local,
                 s_down_local, top_k, capacity=None, gating_mode=_lib.GATING_EXACT, device=0,
                 max_tokens=16384, expert_to_rank=None):
        gate_w = np.asarray(gate_w, np.float32)
        d, e = gate_w.shape
        eloc = e // world
        self.device = device
        self.gate = _lib.Gate(gate_w, gate_b, device)
        if isinstance(q_up_local, _lib.QWeight):
            self.up, self.down = q_up_local, q_down_local
            ffn = q_up_local.N
        else:
            ffn = np.shape(q_up_local)[2]
            self.up = _lib.QWeight(q_up_local, np.asarray(s_up_local, np.float32).reshape(eloc, ffn),
                                   device)
            self.down = _lib.QWeight(q_down_local,
                                     np.asarray(s_down_local, np.float32).reshape(eloc, d), device)
        self.cfg = make_config(d, ffn, e, top_k, capacity, gating_mode)
        uid_buf = (ctypes.c_uint8 * 128).from_buffer_copy(uid)
        place = None
        if expert_to_rank is not None:
            self._place = np.ascontiguousarray(expert_to_rank, dtype=np.int32)
            if self._place.shape != (e,):
                raise ValueError(f"expert_to_rank must have {e} entries")
            place = self._place.ctypes.data
        h = _vp()
        _lib.check(_lib.lib().aem_ep_create(ctypes.byref(self.cfg), rank, world, uid_buf,
                                            self.gate.handle, self.up.handle, self.down.handle,
                                            place, int(max_tokens), ctypes.byref(h)),
                   "aem_ep_create")
        self.handle = h.value
        self.d_model, self.num_experts, self.top_k = d, e, top_k

    def forward(self, x, out=None, out_dtype=None, stream=None):
        import torch
        t = x.shape[0]
        if out is None:
            out = torch.empty((t, self.d_model), dtype=out_dtype or x.dtype, device=x.device)
        _lib.check(_lib.lib().aem_ep_forward(self.handle, x.data_ptr(), _dtype_code(x), t,
                                             out.data_ptr(), _dtype_code(out), _stream_ptr(stream)),
                   "aem_ep_forward")
        return out

    def forward_tolerant(self, x, out=None, out_dtype=None, stream=None):
        """``Router::route_batch_tolerant``: returns ``(out, unit_failed)`` with
        ``unit_failed [k*T]`` uint8 (slot-major); never raises for a peer failure."""
        import torch
        t = x.shape[0]
        if out is None:
            out = torch.empty((t, self.d_model), dtype=out_dtype or x.dtype, device=x.device)
        failed = torch.empty((self.top_k * t,), dtype=torch.uint8, device=x.device)
        _lib.check(_lib.lib().aem_ep_forward_tolerant(self.handle, x.data_ptr(), _dtype_code(x), t,
                                                      out.data_ptr(), _dtype_code(out),
                                                      failed.data_ptr(), _stream_ptr(stream)),
                   "aem_ep_forward_tolerant")
        return out, failed

    def mark_unhealthy(self, rank):
        _lib.check(_lib.lib().aem_ep_mark_unhealthy(self.handle, rank), "aem_ep_mark_unhealthy")

    def health(self, stream=None):
        """Set of ranks left out of later steps (host-marked or found silent)."""
        m = ctypes.c_uint64()
        _lib.check(_lib.lib().aem_ep_health(self.handle, ctypes.byref(m), _stream_ptr(stream)),
                   "aem_ep_health")
        return {r for r in range(64) if (m.value >> r) & 1}

    def set_pipeline(self, mode):
        """Two-half pipeline: -1 automatic (off), 0 off, 1 on (collective)."""
        _lib.check(_lib.lib().aem_ep_set_pipeline(self.handle, int(mode)), "aem_ep_set_pipeline")

    def set_timeout(self, seconds):
        _lib.check(_lib.lib().aem_ep_set_timeout(self.handle, float(seconds)), "aem_ep_set_timeout")

    def profile(self, enable=True):
        _lib.check(_lib.lib().aem_ep_profile(self.handle, 1 if enable else 0), "aem_ep_profile")

    def profile_read(self):
        ms = (ctypes.c_double * _lib.NUM_PHASES)()
        steps = ctypes.c_int64()
        _lib.check(_lib.lib().aem_ep_profile_read(self.handle, ms, ctypes.byref(steps)))
        return dict(zip(_lib.PHASES, list(ms))), steps.value

    def last_routing(self, T, stream=None):
        import torch
        k, e = self.top_k, self.num_experts
        ksel = k + 1 if k < e else k
        dev = torch.device("cuda", self.device)
        idx = torch.empty((T, ksel), dtype=torch.int32, device=dev)
        val = torch.empty((T, k), dtype=torch.float32, device=dev)
        eff = torch.empty((T * k,), dtype=torch.int32, device=dev)
        _lib.check(_lib.lib().aem_ep_last_routing(self.handle, idx.data_ptr(), val.data_ptr(),
                                                  eff.data_ptr(), _stream_ptr(stream)),
                   "aem_ep_last_routing")
        return idx, val, eff

    def close(self):
        if getattr(self, "handle", None):
            _lib.lib().aem_ep_free(self.handle)
            self.handle = None
        for w in ("gate", "up", "down"):
            if getattr(self, w, None) is not None:
                getattr(self, w).close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
