"""ctypes binding of ``libqwen_vpp_native.so`` (declarations: include/qwen_vpp_native.h).

Wire codec, slot rings / physical leases, edge control pages, CUDA IPC
helpers and the peer-to-peer copy issue.  A missing library raises.
"""

import ctypes as ct
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parents[1] / "libqwen_vpp_native.so"

OK, ERR, TIMEOUT, FAILED = 0, -1, -2, -3
SOURCE, DESTINATION = 0, 1
(OP_PRODUCER_RECORDED, OP_TRANSFER_RECORDED, OP_CONSUMER_RECORDED, OP_SOURCE_READ_COMPLETE,
 OP_CONSUMER_COMPLETE, OP_DISCARD_RECEIVED, OP_RELEASE_UNSUBMITTED) = range(7)
STATE_NAMES = ("free", "reserved", "produced", "transferring", "consuming")

_u8p = ct.POINTER(ct.c_uint8)
_vp = ct.c_void_p
_u32, _u64, _i64, _i32 = ct.c_uint32, ct.c_uint64, ct.c_int64, ct.c_int


class QvBoundary(ct.Structure):
    _fields_ = [("epoch", _u64), ("batch_id", _i64), ("edge_sequence", _u64), ("generation", _u64),
                ("src_stage", _u32), ("dst_stage", _u32), ("slot_id", _u32), ("valid_tokens", _u32),
                ("hidden_offset", _u64), ("hidden_bytes", _u64), ("residual_offset", _u64),
                ("residual_bytes", _u64)]

    def as_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_}


class QvKvCopyResult(ct.Structure):
    _fields_ = [("job_id", ct.c_uint64), ("generation", ct.c_uint64), ("bytes", ct.c_uint64),
                ("segments", ct.c_uint64), ("cancelled", ct.c_int32), ("device_ms", ct.c_float),
                ("first_issue_ns", ct.c_uint64), ("last_done_ns", ct.c_uint64)]


class QvTicket(ct.Structure):
    _fields_ = [("ring_id", _u64), ("sequence", _u64), ("generation", _u64), ("slot_id", _u32)]


_LAYOUT = [_u32, _u32, _u32, _u32]
SIGS = {
    "qv_last_error": ([], ct.c_char_p),
    "qv_make_boundary": (_LAYOUT + [_u64, _i64, _u64, _u32, _u32, ct.POINTER(QvBoundary)], _i32),
    "qv_encode_boundary": (_LAYOUT + [ct.POINTER(QvBoundary), _u8p], _i32),
    "qv_decode_boundary": (_LAYOUT + [_u8p, ct.POINTER(QvBoundary)], _i32),
    "qv_match_boundary": (_LAYOUT + [_u8p, _u64, _i64, _u64, _u32, ct.POINTER(QvBoundary)], _i32),
    "qv_rank_boundary_budget": (_LAYOUT + [ct.POINTER(_u64)], _i32),
    "qv_edge_index": ([_u32, _u32, _u32], _i32),
    "qv_ring_create": ([_i32] + _LAYOUT + [_u64, _u32], _vp),
    "qv_ring_destroy": ([_vp], None),
    "qv_ring_try_acquire": ([_vp, ct.POINTER(QvBoundary), ct.POINTER(QvTicket)], _i32),
    "qv_ring_transition": ([_vp, ct.POINTER(QvTicket), _i32], _i32),
    "qv_ring_state": ([_vp, ct.POINTER(QvTicket)], _i32),
    "qv_ring_descriptor": ([_vp, ct.POINTER(QvTicket), ct.POINTER(QvBoundary)], _i32),
    "qv_ring_stop": ([_vp], None),
    "qv_ring_live": ([_vp], _u32),
    "qv_ring_peak_live": ([_vp], _u32),
    "qv_ring_next_sequence": ([_vp], _u64),
    "qv_leases_create": ([_u32], _vp),
    "qv_leases_destroy": ([_vp], None),
    "qv_leases_available": ([_vp], _i32),
    "qv_leases_acquire": ([_vp, ct.POINTER(QvTicket)], _i32),
    "qv_leases_release": ([_vp, _u32, ct.POINTER(QvTicket)], _i32),
    "qv_leases_note_stall": ([_vp], None),
    "qv_leases_live": ([_vp], _u32),
    "qv_leases_peak_live": ([_vp], _u32),
    "qv_leases_stalls": ([_vp], _u64),
    "qv_ctrl_create": ([ct.c_char_p], _vp),
    "qv_ctrl_open": ([ct.c_char_p, ct.c_double], _vp),
    "qv_ctrl_close": ([_vp], None),
    "qv_ctrl_grant": ([_vp, _u64, _u32], _i32),
    "qv_ctrl_wait_grant": ([_vp, _u64, ct.c_double, ct.POINTER(_u32)], _i32),
    "qv_ctrl_publish": ([_vp, _u64, _u8p], _i32),
    "qv_ctrl_wait_published": ([_vp, _u64, ct.c_double, _u8p], _i32),
    "qv_ctrl_peek_published": ([_vp, ct.POINTER(_u64)], _i32),
    "qv_ctrl_fail": ([_vp], None),
    "qv_ctrl_failed": ([_vp], _i32),
    "qv_arena_alloc": ([_i32, _u64, ct.POINTER(_vp), _u8p], _i32),
    "qv_arena_free": ([_i32, _vp], _i32),
    "qv_arena_open": ([_i32, _u8p, ct.POINTER(_vp)], _i32),
    "qv_arena_close": ([_i32, _vp], _i32),
    "qv_ipc_event_create": ([_i32, ct.POINTER(_vp), _u8p], _i32),
    "qv_ipc_event_open": ([_i32, _u8p, ct.POINTER(_vp)], _i32),
    "qv_event_destroy": ([_i32, _vp], _i32),
    "qv_event_query": ([_vp], _i32),
    "qv_copy_message": ([_i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _u64, _u64, _vp, _vp], _i32),
    "qv_stream_wait_event": ([_i32, _vp, _vp], _i32),
    "qv_kvcopy_last_error": ([], ct.c_char_p),
    "qv_kvcopy_create": ([_i32, ct.POINTER(_vp), ct.POINTER(_u64), _i32, _vp, _u64, _u64, _u32, _u32, _i32], _vp),
    "qv_kvcopy_destroy": ([_vp], None),
    "qv_kvcopy_submit": ([_vp, _u64, _u64, ct.POINTER(_i64), _i64, _i32, _vp, ct.POINTER(_i64)], _i32),
    "qv_kvcopy_set_ready": ([_vp, ct.POINTER(_i64), _i64], _i32),
    "qv_kvcopy_cancel": ([_vp, _u64, _u64], _i32),
    "qv_kvcopy_poll": ([_vp, ct.POINTER(QvKvCopyResult), _i32], _i32),
    "qv_kvcopy_snapshot": ([_vp, ct.POINTER(QvKvCopyResult), _i32], _i32),
    "qv_kvcopy_wait": ([_vp, ct.POINTER(_u64), _i32, _u32], _i32),
    "qv_kvcopy_drain": ([_vp, _u32], _i32),
    "qv_kvcopy_close": ([_vp], _i32),
    "qv_kvcopy_plan": ([ct.POINTER(_u64), _i32, _u64, ct.POINTER(_i64), _i64, ct.POINTER(_i64), _i64, _u32,
                        ct.POINTER(_i64), ct.POINTER(_i64), ct.POINTER(_u64)], _i32),
}

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH.name} is not built; run __graft_entry__.build()")
        h = ct.CDLL(str(LIB_PATH))
        for name, (args, res) in SIGS.items():
            fn = getattr(h, name)
            fn.argtypes = args
            fn.restype = res
        _lib = h
    return _lib


class BoundaryError(ValueError):
    pass


def _err():
    return lib().qv_last_error().decode(errors="replace")


def _buf(data=None):
    b = (ct.c_uint8 * 96)()
    if data is not None:
        ct.memmove(b, bytes(data), 96)
    return b


class BoundaryLayout:
    """Capacity (rows per plane), ring slots per edge, ranks and hidden size."""

    def __init__(self, capacity, slots, ranks=4, hidden=5120):
        self.args = (capacity, slots, ranks, hidden)
        self.capacity, self.slots, self.ranks, self.hidden = self.args

    def make(self, epoch, batch, sequence, src_stage, rows):
        d = QvBoundary()
        if lib().qv_make_boundary(*self.args, epoch, batch, sequence, src_stage, rows, ct.byref(d)):
            raise BoundaryError(_err())
        return d

    def encode(self, d):
        out = _buf()
        if lib().qv_encode_boundary(*self.args, ct.byref(d), out):
            raise BoundaryError(_err())
        return bytes(out)

    def decode(self, wire):
        d = QvBoundary()
        if lib().qv_decode_boundary(*self.args, _buf(wire), ct.byref(d)):
            raise BoundaryError(_err())
        return d

    def match(self, wire, epoch, batch, sequence, src_stage):
        d = QvBoundary()
        if lib().qv_match_boundary(*self.args, _buf(wire), epoch, batch, sequence, src_stage, ct.byref(d)):
            raise BoundaryError(_err())
        return d

    def budget(self):
        out = (ct.c_uint64 * self.ranks)()
        if lib().qv_rank_boundary_budget(*self.args, out):
            raise BoundaryError(_err())
        return list(out)


def edge_index(ranks, src, dst):
    v = lib().qv_edge_index(ranks, src, dst)
    if v < 0:
        raise BoundaryError(_err())
    return v


class SlotRing:
    """One edge's logical ring (state machine with generation tickets)."""

    def __init__(self, role, layout, epoch, src_stage):
        self.h = lib().qv_ring_create(role, *layout.args, epoch, src_stage)
        if not self.h:
            raise BoundaryError(_err())

    def try_acquire(self, d):
        t = QvTicket()
        rc = lib().qv_ring_try_acquire(self.h, ct.byref(d), ct.byref(t))
        if rc < 0:
            raise BoundaryError(_err())
        return t if rc == 1 else None

    def transition(self, t, op):
        if lib().qv_ring_transition(self.h, ct.byref(t), op):
            raise BoundaryError(_err())

    def state(self, t):
        rc = lib().qv_ring_state(self.h, ct.byref(t))
        if rc < 0:
            raise BoundaryError(_err())
        return STATE_NAMES[rc]

    def descriptor(self, t):
        d = QvBoundary()
        if lib().qv_ring_descriptor(self.h, ct.byref(t), ct.byref(d)):
            raise BoundaryError(_err())
        return d

    def stop(self):
        lib().qv_ring_stop(self.h)

    @property
    def live(self):
        return lib().qv_ring_live(self.h)

    @property
    def peak_live(self):
        return lib().qv_ring_peak_live(self.h)

    @property
    def next_sequence(self):
        return lib().qv_ring_next_sequence(self.h)

    def close(self):
        if self.h:
            lib().qv_ring_destroy(self.h)
            self.h = None


class PhysicalLeases:
    def __init__(self, slots):
        self.h = lib().qv_leases_create(slots)
        if not self.h:
            raise BoundaryError(_err())

    @property
    def available(self):
        return bool(lib().qv_leases_available(self.h))

    def acquire(self, t):
        rc = lib().qv_leases_acquire(self.h, ct.byref(t))
        if rc < 0:
            raise BoundaryError(_err())
        return rc

    def release(self, physical, t):
        if lib().qv_leases_release(self.h, physical, ct.byref(t)):
            raise BoundaryError(_err())

    def note_stall(self):
        lib().qv_leases_note_stall(self.h)

    @property
    def live(self):
        return lib().qv_leases_live(self.h)

    @property
    def peak_live(self):
        return lib().qv_leases_peak_live(self.h)

    @property
    def stalls(self):
        return lib().qv_leases_stalls(self.h)

    def close(self):
        if self.h:
            lib().qv_leases_destroy(self.h)
            self.h = None


class ControlPage:
    """Shared control page of one directed edge (receiver creates, sender opens)."""

    def __init__(self, name, create, timeout=60.0):
        self.name = name
        raw = name.encode()
        self.h = lib().qv_ctrl_create(raw) if create else lib().qv_ctrl_open(raw, timeout)
        if not self.h:
            raise BoundaryError(_err())

    def grant(self, seq, physical):
        if lib().qv_ctrl_grant(self.h, seq, physical):
            raise BoundaryError("grant failed")

    def wait_grant(self, seq, timeout):
        p = ct.c_uint32()
        rc = lib().qv_ctrl_wait_grant(self.h, seq, timeout, ct.byref(p))
        _check_wait(rc, f"credit for sequence {seq} on {self.name}")
        return p.value

    def publish(self, seq, wire):
        if lib().qv_ctrl_publish(self.h, seq, _buf(wire)):
            raise BoundaryError(f"out-of-order publication of sequence {seq} on {self.name}")

    def wait_published(self, seq, timeout):
        out = _buf()
        rc = lib().qv_ctrl_wait_published(self.h, seq, timeout, out)
        _check_wait(rc, f"publication of sequence {seq} on {self.name}")
        return bytes(out)

    def published(self):
        c = ct.c_uint64()
        lib().qv_ctrl_peek_published(self.h, ct.byref(c))
        return c.value

    def fail(self):
        lib().qv_ctrl_fail(self.h)

    @property
    def failed(self):
        return bool(lib().qv_ctrl_failed(self.h))

    def close(self):
        if self.h:
            lib().qv_ctrl_close(self.h)
            self.h = None


class TransportTimeout(TimeoutError):
    pass


class PeerFailed(RuntimeError):
    pass


def _check_wait(rc, what):
    if rc == OK:
        return
    if rc == TIMEOUT:
        raise TransportTimeout(f"deadline passed waiting for {what}")
    if rc == FAILED:
        raise PeerFailed(f"peer flagged failure while waiting for {what}")
    raise BoundaryError(f"wait for {what} failed ({rc})")


def cuda_check(rc, what):
    if rc:
        raise RuntimeError(f"{what}: CUDA error {rc}")


def arena_alloc(device, nbytes):
    ptr = ct.c_void_p()
    handle = (ct.c_uint8 * 64)()
    cuda_check(lib().qv_arena_alloc(device, nbytes, ct.byref(ptr), handle), "cudaMalloc/cudaIpcGetMemHandle")
    return ptr.value, bytes(handle)


def arena_open(device, handle):
    ptr = ct.c_void_p()
    buf = (ct.c_uint8 * 64).from_buffer_copy(handle)
    cuda_check(lib().qv_arena_open(device, buf, ct.byref(ptr)), "cudaIpcOpenMemHandle")
    return ptr.value


def ipc_event_create(device):
    ev = ct.c_void_p()
    handle = (ct.c_uint8 * 64)()
    cuda_check(lib().qv_ipc_event_create(device, ct.byref(ev), handle), "cudaIpcGetEventHandle")
    return ev.value, bytes(handle)


def ipc_event_open(device, handle):
    ev = ct.c_void_p()
    buf = (ct.c_uint8 * 64).from_buffer_copy(handle)
    cuda_check(lib().qv_ipc_event_open(device, buf, ct.byref(ev)), "cudaIpcOpenEventHandle")
    return ev.value


class DeviceBuffer:
    """Expose a raw device allocation to torch through __cuda_array_interface__."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes // 2,), "typestr": "<u2", "data": (ptr, False),
                                         "version": 3, "strides": None}
