"""Python mirror of the executor C ABI (include/sheaf_b200.h).

Mirrors how Sheaf's runtime drives IREE (sheaf/src/runtime/iree_session.rs):
a process-wide session per GPU, buffers uploaded from host arrays
(buffer_convert.rs:14-123, bf16 rounded to nearest-even on the host), modules
loaded into the session and invoked by "<module>.<function>" with flat leaf
lists (iree_dispatch.rs:172-176), outputs returned as device-resident buffers
that are read back on demand (device_buffer.rs:47-134).
"""
from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np

from . import _lib
from ._lib import ELEM_BF16, ELEM_F16, ELEM_F32, ELEM_I32, lib

NUMPY_OF_ELEM = {ELEM_F32: np.float32, ELEM_I32: np.int32}
ELEM_SIZE = {ELEM_F32: 4, ELEM_I32: 4, ELEM_BF16: 2, ELEM_F16: 2}


class SheafB200Error(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code
        self.message = message


def _check(status) -> None:
    if status:
        L = lib()
        code = L.sb_status_code(status)
        msg = L.sb_status_message(status).decode()
        L.sb_status_free(status)
        raise SheafB200Error(code, msg)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Host-side RNE rounding of f32 to bf16 bit patterns (the conversion
    Sheaf applies before a bf16 upload, sheaf/src/core/dtype.rs:204-216)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    bits = a.view(np.uint32)
    with np.errstate(over="ignore"):
        r = ((bits + np.uint32(0x7FFF) + ((bits >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        r[nan] = (bits[nan] >> np.uint32(16)).astype(np.uint16) | np.uint16(0x40)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


class Session:
    """One executor session on one GPU (sb_session_create)."""

    def __init__(self, device: int = 0):
        self._h = C.c_void_p()
        _check(lib().sb_session_create(device, C.byref(self._h)))
        self.device = device

    @property
    def handle(self):
        return self._h

    def close(self) -> None:
        if self._h:
            lib().sb_session_release(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def synchronize(self, timeout_s: float = 60.0) -> None:
        _check(lib().sb_session_synchronize(self._h, int(timeout_s * 1e9)))

    @property
    def stream(self) -> int:
        return lib().sb_session_stream(self._h) or 0

    def stats(self) -> dict:
        st = _lib.SessionStats()
        _check(lib().sb_session_get_stats(self._h, C.byref(st)))
        return {f: getattr(st, f) for f, _ in st._fields_}

    # -- groups ------------------------------------------------------------
    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = (C.c_char * 128)()
        _check(lib().sb_nccl_unique_id(buf, 128))
        return bytes(buf)

    def join_group(self, nccl_id: bytes, rank: int, world: int) -> None:
        _check(lib().sb_session_join_group(self._h, nccl_id, len(nccl_id), rank, world))

    def leave_group(self, abort: bool = False) -> None:
        """Leaves the data-parallel group, between steps only (no collective of
        this session in flight). abort=True ends the communicator without
        waiting for peers: what the survivors of a departed rank do."""
        _check(lib().sb_session_leave_group(self._h, int(abort)))

    # -- buffers -----------------------------------------------------------
    def upload(self, array, elem: int = ELEM_F32) -> "Buffer":
        """Host array -> new device buffer of element type `elem`."""
        a = np.asarray(array)
        if elem == ELEM_BF16:
            host = f32_to_bf16_bits(a.astype(np.float32))
        elif elem == ELEM_F32:
            host = np.ascontiguousarray(a, dtype=np.float32)
        elif elem == ELEM_I32:
            host = np.ascontiguousarray(a, dtype=np.int32)
        else:
            raise ValueError("unsupported element type")
        shape = (C.c_int64 * max(1, a.ndim))(*a.shape)
        h = C.c_void_p()
        _check(lib().sb_buffer_alloc_copy(self._h, shape, a.ndim, elem, host.ctypes.data_as(C.c_void_p),
                                          host.nbytes, C.byref(h)))
        return Buffer(h)

    def empty(self, shape: Sequence[int], elem: int) -> "Buffer":
        shp = (C.c_int64 * max(1, len(shape)))(*shape)
        h = C.c_void_p()
        _check(lib().sb_buffer_alloc(self._h, shp, len(shape), elem, C.byref(h)))
        return Buffer(h)

    # -- modules -----------------------------------------------------------
    def load_stablehlo(self, text: str) -> str:
        data = text.encode()
        name = C.c_char_p()
        _check(lib().sb_module_load_stablehlo(self._h, data, len(data), C.byref(name)))
        return name.value.decode()

    def describe(self, module: str) -> str:
        buf = C.create_string_buffer(4096)
        _check(lib().sb_module_describe(self._h, module.encode(), buf, 4096))
        return buf.value.decode()

    def create_gpt_vag(self, name: str, *, n_layer, n_head, n_embd, block_size, vocab_size, batch, seq,
                       elem=ELEM_BF16) -> str:
        cfg = _lib.GptConfig(n_layer, n_head, n_embd, block_size, vocab_size, batch, seq, elem)
        _check(lib().sb_module_create_gpt_vag(self._h, name.encode(), C.byref(cfg)))
        return name

    def create_gpt_train(self, name: str, *, n_layer, n_head, n_embd, block_size, vocab_size, batch, seq,
                         elem=ELEM_BF16, b1=0.9, b2=0.95, eps=1e-8, weight_decay=0.1, max_norm=1.0) -> str:
        """nanoGPT train-step module (value_and_grad + clip-by-global-norm +
        AdamW); the defaults are examples/nanogpt/train.shf's constants."""
        cfg = _lib.GptConfig(n_layer, n_head, n_embd, block_size, vocab_size, batch, seq, elem)
        opt = _lib.AdamwConfig(b1, b2, eps, weight_decay, max_norm)
        _check(lib().sb_module_create_gpt_train(self._h, name.encode(), C.byref(cfg), C.byref(opt)))
        return name

    def create_gpt_sampler(self, name: str, *, n_layer, n_head, n_embd, block_size, vocab_size, batch,
                           n_new, top_k=200, temperature=0.8, elem=ELEM_BF16) -> str:
        """nanoGPT sampling module (generate-token + slide-window repeated
        n_new times); the defaults are examples/nanogpt/sample.shf's top-k 200
        and temperature 0.8. Function "generate": leaves, ids [batch,
        block_size], keys [batch, 4] -> tokens, ids', keys', step logits."""
        cfg = _lib.GptConfig(n_layer, n_head, n_embd, block_size, vocab_size, batch, block_size, elem)
        smp = _lib.SamplerConfig(n_new, top_k, temperature)
        _check(lib().sb_module_create_gpt_sampler(self._h, name.encode(), C.byref(cfg), C.byref(smp)))
        return name

    # -- checkpoints (io "save" / io "load", builtins/safetensors.rs) ----------
    def save_safetensors(self, path: str, tree) -> None:
        """Writes a pytree of device buffers (dicts, lists, Buffer leaves) as
        the reference's save_safetensors does: dot-separated keys (dict keys,
        list indices), sorted; each buffer's bytes go straight to the file."""
        items = _flatten_tree(tree)
        for k, v in items:
            if not isinstance(v, Buffer):
                raise TypeError(f"checkpoint leaf {k!r} is not a device buffer")
        n = len(items)
        keys = (C.c_char_p * max(1, n))(*[k.encode() for k, _ in items])
        bufs = (C.c_void_p * max(1, n))(*[v._h for _, v in items])
        _check(lib().sb_safetensors_save(self._h, str(path).encode(), keys, bufs, n))

    def load_safetensors(self, path: str, nested: bool = True):
        """Reads every tensor of a safetensors file into a device buffer;
        with `nested`, dot-separated keys become dicts and contiguous numeric
        siblings lists (load_safetensors's nest_flat_keys)."""
        f = C.c_void_p()
        _check(lib().sb_safetensors_open(str(path).encode(), C.byref(f)))
        flat = {}
        try:
            for i in range(lib().sb_safetensors_count(f)):
                key = lib().sb_safetensors_key(f, i).decode()
                h = C.c_void_p()
                _check(lib().sb_safetensors_read(self._h, f, i, C.byref(h)))
                flat[key] = Buffer(h)
        finally:
            lib().sb_safetensors_close(f)
        return _nest_keys(flat) if nested else flat

    # -- data path (train.shf get-batch, random-split) -----------------------
    def random_split(self, key: "Buffer", n: int = 2) -> "Buffer":
        """Child keys [n, 4] of a key buffer [4] (f32 limbs)."""
        out = self.empty((n, 4), ELEM_F32)
        rc = lib().sb_op_random_split(C.c_void_p(key.device_ptr), n, C.c_void_p(out.device_ptr),
                                      C.c_void_p(self.stream))
        if rc:
            raise SheafB200Error(3, f"random_split failed ({rc})")
        return out

    def get_batch(self, data: "Buffer", key: "Buffer", block: int, batch: int) -> tuple["Buffer", "Buffer"]:
        """get-batch on the device: x, y [batch, block] f32 ids from the f32
        token array `data` at starts drawn from `key` (train.shf:15-21)."""
        (n,) = data.shape
        x = self.empty((batch, block), ELEM_F32)
        y = self.empty((batch, block), ELEM_F32)
        rc = lib().sb_op_get_batch(C.c_void_p(data.device_ptr), n, C.c_void_p(key.device_ptr), block, batch,
                                   C.c_void_p(x.device_ptr), C.c_void_p(y.device_ptr), C.c_void_p(self.stream))
        if rc:
            raise SheafB200Error(3, f"get_batch failed ({rc})")
        return x, y

    def call(self, qualified_name: str, inputs: Sequence["Buffer"], max_outputs: int = 1024) -> "Outputs":
        arr = (C.c_void_p * max(1, len(inputs)))(*[b._h for b in inputs])
        outs = (C.c_void_p * max_outputs)()
        n = C.c_size_t()
        _check(lib().sb_call(self._h, qualified_name.encode(), arr, len(inputs), outs, max_outputs, C.byref(n)))
        return Outputs(outs, n.value)


# ---- leaving a data-parallel group between steps -------------------------
# An all-reduce enqueued on the GPU waits for every peer without a limit, so a
# rank may leave only between steps. It announces its departure in the
# process group's key-value store before the step-boundary barrier; after
# that barrier every survivor reads the announcements, before it enqueues the
# next step, and ends its communicator with Session.leave_group(abort=True).

def _departure_key(rank: int) -> str:
    return f"sheaf_b200/departed/{rank}"


def announce_departure(store, rank: int) -> None:
    """Marks `rank` as leaving after the current step (a torch.distributed
    Store, e.g. the default process group's)."""
    store.set(_departure_key(rank), "1")


def departed_ranks(store, world: int) -> list[int]:
    """Ranks that announced their departure (read after the step-boundary
    barrier, so an announcement made before it is always seen)."""
    return [r for r in range(world) if store.check([_departure_key(r)])]


def validate_stablehlo(text: str) -> str:
    """Parses and plans a StableHLO module on the host (no device needed);
    returns the summary or raises SheafB200Error (UNIMPLEMENTED = 12)."""
    data = text.encode()
    buf = C.create_string_buffer(8192)
    _check(lib().sb_stablehlo_validate(data, len(data), buf, 8192))
    return buf.value.decode()


def _flatten_tree(tree, prefix: str = "") -> list:
    """(key, leaf) pairs: dict keys in sorted order, list items by index,
    joined with '.'; a leaf at the root is named 'tensor'."""
    if isinstance(tree, dict):
        out = []
        for k in sorted(tree):
            out += _flatten_tree(tree[k], f"{prefix}.{k}" if prefix else str(k))
        return out
    if isinstance(tree, (list, tuple)):
        out = []
        for i, v in enumerate(tree):
            out += _flatten_tree(v, f"{prefix}.{i}" if prefix else str(i))
        return out
    return [(prefix or "tensor", tree)]


def _nest_keys(flat: dict):
    root: dict = {}
    for key in sorted(flat):
        node = root
        segs = key.split(".")
        for seg in segs[:-1]:
            node = node.setdefault(seg, {})
        node[segs[-1]] = flat[key]

    def lists(node):
        if not isinstance(node, dict):
            return node
        node = {k: lists(v) for k, v in node.items()}
        if node and all(k.isdigit() for k in node) and max(int(k) for k in node) + 1 == len(node):
            return [node[str(i)] for i in range(len(node))]
        return node
    return lists(root)


class Outputs(Sequence):
    """The buffers a call returned, in order (loss first, then the gradient
    leaves, for a value_and_grad). An entry becomes a Buffer, which then owns
    it, when first read; the entries never read are released together (one
    foreign call) when the sequence is dropped."""

    __slots__ = ("_arr", "_n", "_bufs")

    def __init__(self, arr, n: int):
        self._arr = arr
        self._n = n
        self._bufs: list = [None] * n

    def __len__(self) -> int:
        return self._n

    def __getitem__(self, i):
        if isinstance(i, slice):
            return [self[j] for j in range(*i.indices(self._n))]
        if i < 0:
            i += self._n
        if not 0 <= i < self._n:
            raise IndexError(i)
        b = self._bufs[i]
        if b is None:
            b = Buffer(C.c_void_p(self._arr[i]))
            self._arr[i] = None
            self._bufs[i] = b
        return b

    def release(self) -> None:
        if self._arr is not None:
            lib().sb_buffer_release_many(self._arr, self._n)
            self._arr = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class Buffer:
    """A device buffer view (sb_buffer); released when garbage collected."""

    def __init__(self, handle):
        self._h = handle
        self._meta = None  # (shape, elem, nbytes): fixed for a buffer's life

    def release(self) -> None:
        if self._h:
            lib().sb_buffer_release(self._h)
            self._h = None

    def _info(self):
        if self._meta is None:
            L = lib()
            shape = tuple(L.sb_buffer_dim(self._h, i) for i in range(L.sb_buffer_rank(self._h)))
            self._meta = (shape, L.sb_buffer_elem_type(self._h), L.sb_buffer_byte_length(self._h))
        return self._meta

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass

    @property
    def shape(self) -> tuple[int, ...]:
        return self._info()[0]

    @property
    def elem(self) -> int:
        return self._info()[1]

    @property
    def nbytes(self) -> int:
        return self._info()[2]

    @property
    def device_ptr(self) -> int:
        return lib().sb_buffer_device_ptr(self._h) or 0

    def write(self, host: np.ndarray) -> None:
        h = np.ascontiguousarray(host)
        _check(lib().sb_buffer_h2d(self._h, h.ctypes.data_as(C.c_void_p), h.nbytes))

    def to_host(self, timeout_s: float = 60.0) -> np.ndarray:
        """D2H + widening to f32 (as device_buffer.rs to_host does)."""
        e = self.elem
        n = self.nbytes
        if e in (ELEM_BF16, ELEM_F16):
            raw = np.empty(n // 2, dtype=np.uint16)
        elif e == ELEM_I32:
            raw = np.empty(n // 4, dtype=np.int32)
        else:
            raw = np.empty(n // 4, dtype=np.float32)
        _check(lib().sb_buffer_d2h(self._h, raw.ctypes.data_as(C.c_void_p), n, int(timeout_s * 1e9)))
        if e == ELEM_BF16:
            out = bf16_bits_to_f32(raw)
        elif e == ELEM_F16:
            out = raw.view(np.float16).astype(np.float32)
        else:
            out = raw
        return out.reshape(self.shape)
