"""ctypes binding of ``libaethermoe.so`` (declared in ``include/aem.h``).

Loading fails loudly: there is no CPU fallback for any entry point.  Status
codes become exceptions the way the reference reports errors
(``ValueError`` for bad arguments, ``fused_gating_metal.py:380-388``,
``quantized_gemm.py:204-205``; ``RuntimeError`` otherwise).
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libaethermoe.so")

AEM_OK, AEM_EINVAL, AEM_ECUDA, AEM_ENCCL, AEM_ETIMEOUT, AEM_ENOMEM, AEM_EUNSUPPORTED, AEM_EDEVICE = range(8)
F32, BF16 = 0, 1
GATING_EXACT, GATING_FAST, GATING_CERTIFIED = 0, 1, 2
CAPACITY_UNLIMITED = (1 << 64) - 1
MAX_EXPERTS = 256
MAX_TOPK = 64

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_u64 = ctypes.c_uint64


class AemError(RuntimeError):
    """A failed library call (CUDA, NCCL, timeout, in-kernel check)."""

    def __init__(self, status, message):
        super().__init__(f"[aem status {status}] {message}")
        self.status = status


class AemTimeout(AemError):
    pass


class MoeConfig(ctypes.Structure):
    _fields_ = [("d_model", _i64), ("d_ffn", _i64), ("num_experts", _int), ("top_k", _int),
                ("capacity", _u64), ("gating_mode", _int)]


class SeqSlice(ctypes.Structure):
    """``aem_seq_slice``: one sequence's rows in a continuous-batching iteration."""
    _fields_ = [("seq_id", ctypes.c_uint64), ("x", ctypes.c_void_p), ("out", ctypes.c_void_p),
                ("tokens", ctypes.c_int64)]


EP_MAX_RANKS = 64
METRIC_MOE_STEP, METRIC_EP_STEP = 0, 1


class MetricStats(ctypes.Structure):
    """``aem_metric_stats`` (the reference's MetricStats, src/core/telemetry.hpp:35-42)."""
    _fields_ = [("count", ctypes.c_uint64), ("mean_ns", ctypes.c_double),
                ("p50_ns", ctypes.c_double), ("p95_ns", ctypes.c_double),
                ("p99_ns", ctypes.c_double), ("max_ns", ctypes.c_double)]

    def as_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_}


class EpPeerPlan(ctypes.Structure):
    """``aem_ep_peer_plan``: where one rank's rows go in one peer-memory exchange."""
    _fields_ = [("ok", ctypes.c_int32), ("units_in", ctypes.c_int32),
                ("units_in_a", ctypes.c_int32),
                ("pairs_in", ctypes.c_int32), ("pairs_out", ctypes.c_int32),
                ("dst_unit_off", (ctypes.c_int32 * 256) * 2),
                ("dst_pair_off", ctypes.c_int32 * EP_MAX_RANKS),
                ("send_pair_off", ctypes.c_int32 * EP_MAX_RANKS),
                ("send_pair_a", ctypes.c_int32 * EP_MAX_RANKS),
                ("recv_pair_off", ctypes.c_int32 * (EP_MAX_RANKS + 1)),
                ("recv_pair_a", ctypes.c_int32 * EP_MAX_RANKS),
                ("ret_off", ctypes.c_int32 * EP_MAX_RANKS)]


def ep_payload_words(E, R):
    """``AEM_EP_PAYLOAD(E, R)``: int32 words of one rank's exchange payload."""
    return (2 * E + 3 + 2 * R + 3) & ~3


_SIGS = {
    "aem_last_error": (ctypes.c_char_p, []),
    "aem_version": (ctypes.c_char_p, []),
    "aem_device_count": (_int, []),
    "aem_device_status": (_int, [_vp]),
    "aem_context_create": (_int, [_int, ctypes.POINTER(_vp)]),
    "aem_context_destroy": (_int, [_vp]),
    "aem_context_stream": (_vp, [_vp]),
    "aem_gate_pack": (_int, [_vp, _vp, _i64, _i64, _int, ctypes.POINTER(_vp)]),
    "aem_gate_free": (_int, [_vp]),
    "aem_gate_fallback_rows": (_int, [_vp, ctypes.POINTER(_i64)]),
    "aem_gating": (_int, [_vp, _vp, _int, _i64, _int, _int, _int, _vp, _vp, _vp]),
    "aem_gating_host": (_int, [_vp, _vp, _vp, _int, _i64, _int, _int, _int, _vp, _vp]),
    "aem_quantize_int8": (_int, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "aem_quantize_int8_host": (_int, [_vp, _vp, _i64, _i64, _vp, _vp]),
    "aem_qweight_pack": (_int, [_vp, _vp, _i64, _i64, _i64, _int, ctypes.POINTER(_vp)]),
    "aem_qweight_pack_device": (_int, [_vp, _vp, _i64, _i64, _i64, _vp, ctypes.POINTER(_vp)]),
    "aem_qweight_free": (_int, [_vp]),
    "aem_qweight_shape": (_int, [_vp, ctypes.POINTER(_i64), ctypes.POINTER(_i64),
                                 ctypes.POINTER(_i64)]),
    "aem_qgemm": (_int, [_vp, _i64, _vp, _int, _i64, _vp, _vp]),
    "aem_qgemm_host": (_int, [_vp, _vp, _i64, _vp, _int, _i64, _vp]),
    "aem_grouped_qgemm": (_int, [_vp, _vp, _int, _vp, _i64, _vp, _int, _i64, _int, _int, _vp, _vp,
                                 _int, _int, _vp]),
    "aem_capacity_route_workspace": (ctypes.c_size_t, [_i64, _int]),
    "aem_capacity_route": (_int, [_vp, _vp, _vp, _i64, _int, _u64, _vp, _vp, ctypes.c_size_t,
                                  _vp]),
    "aem_moe_create": (_int, [ctypes.POINTER(MoeConfig), _vp, _vp, _vp, ctypes.POINTER(_vp)]),
    "aem_moe_free": (_int, [_vp]),
    "aem_moe_forward": (_int, [_vp, _vp, _int, _i64, _vp, _int, _vp]),
    "aem_moe_forward_host": (_int, [_vp, _vp, _vp, _int, _i64, _vp, _int]),
    "aem_moe_last_routing": (_int, [_vp, _vp, _vp, _vp, _vp]),
    "aem_ep_plan_bases": (_int, [_vp, _int, _int, _int, _int, _vp]),
    "aem_ep_unique_id": (_int, [_vp]),
    "aem_ep_plan_exchange": (_int, [_vp, _int, _int, _int, _vp, _vp, _vp, _vp, _vp]),
    "aem_ep_plan_peer": (_int, [_vp, _int, _int, _int, _u64, _i64, _i64, _i64,
                                ctypes.POINTER(EpPeerPlan), _vp]),
    "aem_ep_plan_peer_device": (_int, [_vp, _int, _int, _int, _u64, _i64, _i64, _i64, _vp, _vp,
                                       _vp]),
    "aem_ep_forward_tolerant": (_int, [_vp, _vp, _int, _i64, _vp, _int, _vp, _vp]),
    "aem_ep_mark_unhealthy": (_int, [_vp, _int]),
    "aem_ep_health": (_int, [_vp, ctypes.POINTER(_u64), _vp]),
    "aem_ep_set_timeout": (_int, [_vp, ctypes.c_double]),
    "aem_ep_set_pipeline": (_int, [_vp, _int]),
    "aem_ep_create": (_int, [ctypes.POINTER(MoeConfig), _int, _int, _vp, _vp, _vp, _vp, _vp,
                             _i64, ctypes.POINTER(_vp)]),
    "aem_ep_free": (_int, [_vp]),
    "aem_ep_forward": (_int, [_vp, _vp, _int, _i64, _vp, _int, _vp]),
    "aem_ep_forward_host": (_int, [_vp, _vp, _vp, _int, _i64, _vp, _int]),
    "aem_ep_submit_host": (_int, [_vp, _vp, _vp, _int, _i64, _vp, _int,
                                  ctypes.POINTER(ctypes.c_uint64)]),
    "aem_moe_submit_host": (_int, [_vp, _vp, _vp, _int, _i64, _vp, _int,
                                   ctypes.POINTER(ctypes.c_uint64)]),
    "aem_context_wait": (_int, [_vp, ctypes.c_uint64]),
    "aem_ep_last_routing": (_int, [_vp, _vp, _vp, _vp, _vp]),
    "aem_capacity_route_static": (_int, [_vp, _vp, _vp, _i64, _int, _u64, _vp, _vp]),
    "aem_kernel_launches": (ctypes.c_uint64, []),
    "aem_moe_profile": (_int, [_vp, _int]),
    "aem_moe_set_hidden_dtype": (_int, [_vp, _int]),
    "aem_set_gemm_pairs": (_int, [_int]),
    "aem_set_gemm_tmem_a": (_int, [_int]),
    "aem_moe_profile_read": (_int, [_vp, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_i64)]),
    "aem_ep_profile": (_int, [_vp, _int]),
    "aem_ep_profile_read": (_int, [_vp, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_i64)]),
    "aem_moe_forward_slices": (_int, [_vp, ctypes.POINTER(SeqSlice), _int, _int, _int, _vp]),
    "aem_telemetry_enable": (None, [_int]),
    "aem_telemetry_enabled": (_int, []),
    "aem_telemetry_snapshot": (_int, [_int, ctypes.POINTER(MetricStats), ctypes.POINTER(_u64)]),
    "aem_telemetry_reset": (_int, []),
    "aem_metric_stats_of": (_int, [_vp, _i64, ctypes.POINTER(MetricStats)]),
}
NUM_PHASES = 8
PHASES = ["gating", "route", "up_gemm", "down_gemm", "combine", "dispatch", "return", "exchange"]

_lib = None
_lock = threading.Lock()


def lib():
    """The loaded library (raises if it was not built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is missing: build it with `python -m aethermoe_b200.build` "
                        "(there is no CPU fallback)")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in _SIGS.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def exported_symbols():
    return list(_SIGS)


def last_error():
    return lib().aem_last_error().decode(errors="replace")


def check(status, what=""):
    """Raises the exception matching an aem_status."""
    if status == AEM_OK:
        return
    msg = last_error()
    if what:
        msg = f"{what}: {msg}"
    if status == AEM_EINVAL:
        raise ValueError(msg)
    if status == AEM_ETIMEOUT:
        raise AemTimeout(status, msg)
    raise AemError(status, msg)


def device_count():
    return lib().aem_device_count()


# ------------------------------------------------------------------ contexts
_contexts = {}


def context(device=0):
    """Per-device staging context for the *_host calls (created lazily)."""
    c = _contexts.get(device)
    if c is None:
        h = _vp()
        check(lib().aem_context_create(device, ctypes.byref(h)), "aem_context_create")
        c = h.value
        _contexts[device] = c
    return c


class Gate:
    """Packed gating layer (device-resident [D/4][Epad][4] copy of W [D, E])."""

    def __init__(self, gate_weight, gate_bias, device=0):
        import numpy as np
        w = np.ascontiguousarray(gate_weight, dtype=np.float32)
        if w.ndim != 2:
            raise ValueError("gate_weight must be [D, E]")
        d, e = w.shape
        b = None if gate_bias is None else np.ascontiguousarray(gate_bias, dtype=np.float32).reshape(-1)
        if b is not None and b.shape[0] != e:
            raise ValueError(f"gate_bias has {b.shape[0]} entries, expected {e}")
        h = _vp()
        check(lib().aem_gate_pack(w.ctypes.data, None if b is None else b.ctypes.data, d, e,
                                  device, ctypes.byref(h)), "aem_gate_pack")
        self.handle = h.value
        self.D, self.E, self.device = d, e, device

    def fallback_rows(self):
        """Rows of CERTIFIED-mode calls recomputed with the EXACT arithmetic so far."""
        n = _i64()
        check(lib().aem_gate_fallback_rows(self.handle, ctypes.byref(n)), "aem_gate_fallback_rows")
        return n.value

    def close(self):
        if getattr(self, "handle", None):
            lib().aem_gate_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class QWeight:
    """Packed INT8 weight groups: q [G][K][N] int8 + scale [G][N] -> device [G][N][K]."""

    def __init__(self, q, scale, device=0):
        import numpy as np
        q = np.ascontiguousarray(q, dtype=np.int8)
        if q.ndim == 2:
            q = q[None]
        g, k, n = q.shape
        s = np.ascontiguousarray(scale, dtype=np.float32).reshape(g, n)
        h = _vp()
        check(lib().aem_qweight_pack(q.ctypes.data, s.ctypes.data, g, k, n, device,
                                     ctypes.byref(h)), "aem_qweight_pack")
        self.handle = h.value
        self.G, self.K, self.N, self.device = g, k, n, device

    def close(self):
        if getattr(self, "handle", None):
            lib().aem_qweight_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DeviceQWeight(QWeight):
    """Packed INT8 weight groups built from DEVICE tensors (torch CUDA):
    ``q [G, K, N]`` int8 and ``scale [G, N]`` float32 (stream-ordered pack)."""

    def __init__(self, q, scale, stream=None):  # noqa: D401 - torch tensors
        import torch
        if q.dim() == 2:
            q = q.unsqueeze(0)
        g, k, n = q.shape
        q = q.contiguous()
        scale = scale.reshape(g, n).contiguous().float()
        s = stream or torch.cuda.current_stream(q.device)
        h = _vp()
        check(lib().aem_qweight_pack_device(q.data_ptr(), scale.data_ptr(), g, k, n,
                                            ctypes.c_void_p(s.cuda_stream), ctypes.byref(h)),
              "aem_qweight_pack_device")
        s.synchronize()
        self.handle = h.value
        self.G, self.K, self.N, self.device = g, k, n, q.device.index


def quantize_device(w, stream=None):
    """Bit-exact per-output-column INT8 quantisation of a float32 CUDA tensor
    ``w [K, N]`` -> ``(q int8 [K, N], scale float32 [N])`` (aem_quantize_int8)."""
    import torch
    w = w.contiguous().float()
    k, n = w.shape
    q = torch.empty((k, n), dtype=torch.int8, device=w.device)
    s = torch.empty((n,), dtype=torch.float32, device=w.device)
    st = stream or torch.cuda.current_stream(w.device)
    check(lib().aem_quantize_int8(w.data_ptr(), k, n, q.data_ptr(), s.data_ptr(),
                                  ctypes.c_void_p(st.cuda_stream)), "aem_quantize_int8")
    return q, s


def telemetry_enable(enabled=True):
    """Per-step device-time telemetry of the MoE layers (process-wide switch)."""
    lib().aem_telemetry_enable(1 if enabled else 0)


def telemetry_snapshot(metric=METRIC_MOE_STEP):
    """``(stats dict, dropped)`` of every completed step of ``metric`` so far."""
    st = MetricStats()
    dropped = ctypes.c_uint64()
    check(lib().aem_telemetry_snapshot(metric, ctypes.byref(st), ctypes.byref(dropped)),
          "aem_telemetry_snapshot")
    return st.as_dict(), dropped.value


def telemetry_reset():
    check(lib().aem_telemetry_reset(), "aem_telemetry_reset")


def metric_stats_of(latencies_ns):
    """Nearest-rank statistics of host latencies (the snapshot's arithmetic)."""
    import numpy as np
    a = np.ascontiguousarray(latencies_ns, dtype=np.uint64)
    st = MetricStats()
    check(lib().aem_metric_stats_of(a.ctypes.data if a.size else None, a.size, ctypes.byref(st)),
          "aem_metric_stats_of")
    return st.as_dict()
