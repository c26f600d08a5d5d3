"""Host mirror of the entity-encoder policy ABI (include/ow_policy.h).

    pol = EncoderPolicy(cfg, weights)                 # host IO, synchronous
    logits, value, actions = pol.forward(features, counts, seed=0)

    pol = EncoderPolicy(cfg, weights, io="device")    # device IO, async on pol's stream
    pol.forward_device(feat_ptr, counts_ptr, batch, logits_ptr, value_ptr, actions_ptr)
    pol.synchronize()
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from .presets import DTYPE, IO, PRECISION, PolicyConfig


def to_config_c(cfg: PolicyConfig, io: str = "host", batch_capacity: int | None = None) -> _lib.PolicyConfigC:
    c = _lib.PolicyConfigC()
    c.batch_capacity = int(batch_capacity if batch_capacity is not None else cfg.batch)
    c.n_entities, c.features, c.d_model, c.heads = cfg.n_entities, cfg.features, cfg.d_model, cfg.heads
    c.ffn, c.layers, c.actions = cfg.ffn, cfg.layers, cfg.actions
    c.precision = PRECISION[cfg.precision]
    c.sample_actions = 1 if cfg.sample_actions else 0
    c.logits_dtype, c.value_dtype = DTYPE[cfg.logits_dtype], DTYPE[cfg.value_dtype]
    c.io = IO[io]
    return c


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


class EncoderPolicy:
    def __init__(self, cfg: PolicyConfig, weights: np.ndarray | None, device: int = 0, stream: int | None = None,
                 io: str = "host", batch_capacity: int | None = None):
        """weights None: the handle holds zero weights until broadcast_from() fills them."""
        self.lib = _lib.load_library()
        self.cfg = cfg
        self.io = io
        self.device = device
        self.ccfg = to_config_c(cfg, io, batch_capacity)
        h = C.c_void_p()
        if weights is None:
            n = C.c_size_t()
            _lib.check("ow_policy_weight_count", self.lib.ow_policy_weight_count(C.byref(self.ccfg), C.byref(n)))
            _lib.check("ow_policy_create", self.lib.ow_policy_create(
                C.byref(self.ccfg), None, n.value, device, stream, C.byref(h)))
        else:
            w = np.ascontiguousarray(weights, dtype=np.float32)
            _lib.check("ow_policy_create", self.lib.ow_policy_create(
                C.byref(self.ccfg), w.ctypes.data_as(_lib.FP), w.size, device, stream, C.byref(h)))
        self.handle = h

    def broadcast_from(self, comm: "Comm", root: int = 0) -> float:
        """Every rank calls this: the root's device weights replace this handle's (one ncclBroadcast of the
        packed weight arena). Returns this rank's broadcast device time in ms."""
        ms = C.c_float()
        _lib.check("ow_policy_broadcast_weights_comm", self.lib.ow_policy_broadcast_weights_comm(
            self.handle, comm.handle, int(root), C.byref(ms)))
        return float(ms.value)

    def set_weights(self, weights: np.ndarray) -> None:
        w = np.ascontiguousarray(weights, dtype=np.float32)
        _lib.check("ow_policy_set_weights", self.lib.ow_policy_set_weights(self.handle, w.ctypes.data_as(_lib.FP), w.size))

    def forward(self, features: np.ndarray, counts: np.ndarray, seed: int = 0):
        """Host IO forward: returns (logits f32 [B,N,P], value f32 [B], actions int32 [B,N])."""
        assert self.io == "host"
        cfg = self.cfg
        f = np.ascontiguousarray(features, dtype=np.float32)
        c = np.ascontiguousarray(counts, dtype=np.int32)
        B = c.shape[0]
        if f.shape != (B, cfg.n_entities, cfg.features):
            raise ValueError(f"features shape {f.shape} != {(B, cfg.n_entities, cfg.features)}")
        lb = cfg.logits_dtype == "bf16"
        vb = cfg.value_dtype == "bf16"
        logits = np.empty((B, cfg.n_entities, cfg.actions), dtype=np.uint16 if lb else np.float32)
        value = np.empty((B,), dtype=np.uint16 if vb else np.float32)
        actions = np.empty((B, cfg.n_entities), dtype=np.int32)
        _lib.check("ow_policy_forward", self.lib.ow_policy_forward(
            self.handle, f.ctypes.data, c.ctypes.data, B, logits.ctypes.data, value.ctypes.data,
            actions.ctypes.data, C.c_uint64(seed)))
        if lb:
            logits = bf16_bits_to_f32(logits)
        if vb:
            value = bf16_bits_to_f32(value)
        return logits, value, actions

    def forward_raw(self, features_ptr, counts_ptr, batch: int, logits_ptr, value_ptr, actions_ptr,
                    seed: int = 0) -> None:
        """Forward on raw pointers (host pointers in host IO mode, device pointers in device IO mode)."""
        _lib.check("ow_policy_forward", self.lib.ow_policy_forward(
            self.handle, features_ptr, counts_ptr, int(batch), logits_ptr, value_ptr, actions_ptr, C.c_uint64(seed)))

    forward_device = forward_raw

    def submit_raw(self, features_ptr, counts_ptr, batch: int, logits_ptr, value_ptr, actions_ptr,
                   seed: int = 0) -> int:
        """Host-IO pipelined forward: enqueue upload, forward and download; returns a ticket.
        The host buffers (pinned for overlap) must stay valid until wait(ticket)."""
        t = C.c_int64()
        _lib.check("ow_policy_submit", self.lib.ow_policy_submit(
            self.handle, features_ptr, counts_ptr, int(batch), logits_ptr, value_ptr, actions_ptr, C.c_uint64(seed),
            C.byref(t)))
        return t.value

    def wait(self, ticket: int) -> None:
        """Blocks until the submission's outputs are in its host buffers; raises on its errors."""
        _lib.check("ow_policy_wait", self.lib.ow_policy_wait(self.handle, C.c_int64(ticket)))

    def synchronize(self) -> None:
        _lib.check("ow_policy_synchronize", self.lib.ow_policy_synchronize(self.handle))

    def device_weights(self) -> tuple[int, int]:
        p, n = C.c_void_p(), C.c_size_t()
        _lib.check("ow_policy_device_weights", self.lib.ow_policy_device_weights(self.handle, C.byref(p), C.byref(n)))
        return p.value, n.value

    def launches_per_forward(self) -> int:
        n = C.c_int32()
        _lib.check("ow_policy_launches_per_forward", self.lib.ow_policy_launches_per_forward(self.handle, C.byref(n)))
        return n.value

    def profile_begin(self, max_forwards: int) -> None:
        _lib.check("ow_policy_profile_begin", self.lib.ow_policy_profile_begin(self.handle, int(max_forwards)))

    def profile_end(self) -> dict[str, tuple[int, float]]:
        """{kernel name: (launches, total device ms)} since profile_begin."""
        buf = (_lib.KernelTimingC * 64)()
        n = C.c_int32()
        _lib.check("ow_policy_profile_end", self.lib.ow_policy_profile_end(self.handle, buf, 64, C.byref(n)))
        return {buf[i].name.decode(): (buf[i].launches, buf[i].total_ms) for i in range(n.value)}

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.ow_policy_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


class Comm:
    """NCCL communicator for the weight broadcast (include/ow_policy.h, "Weight broadcast over NCCL").

        uid = Comm.unique_id()                  # on one rank; share the 128 bytes over any channel
        comm = Comm(uid, nranks, rank, device)  # on every rank
        pol.broadcast_from(comm, root=0)
    """

    def __init__(self, uid: bytes, nranks: int, rank: int, device: int):
        self.lib = _lib.load_library()
        buf = C.create_string_buffer(bytes(uid), 128)
        h = C.c_void_p()
        _lib.check("ow_comm_init_rank", self.lib.ow_comm_init_rank(buf, 128, int(nranks), int(rank), int(device),
                                                                    C.byref(h)))
        self.handle = h
        self.rank, self.nranks, self.device = int(rank), int(nranks), int(device)

    @staticmethod
    def unique_id() -> bytes:
        lib = _lib.load_library()
        buf = C.create_string_buffer(128)
        _lib.check("ow_comm_unique_id", lib.ow_comm_unique_id(buf, 128))
        return buf.raw

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.ow_comm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def broadcast_weights_all(policies: list["EncoderPolicy"]) -> None:
    """One process, one handle per GPU: policies[0]'s weights go to the others (ow_policy_broadcast_weights)."""
    lib = _lib.load_library()
    arr = (C.c_void_p * len(policies))(*[p.handle.value for p in policies])
    _lib.check("ow_policy_broadcast_weights", lib.ow_policy_broadcast_weights(arr, len(policies)))


def nccl_version() -> int:
    lib = _lib.load_library()
    v = C.c_int()
    _lib.check("ow_nccl_version", lib.ow_nccl_version(C.byref(v)))
    return v.value
