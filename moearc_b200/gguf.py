"""A GGUF model file, read through the library's moearc_x_gguf_* entry points.

The host mirror of the reference's model reader (crates/moearc-model/src/gguf.rs, the header
parse, and tensors.rs, the zero-copy tensor views and `slice_last_dim` for one expert of a
stacked bank). The file is mapped by the library; a tensor's bytes are a view of the mapping,
valid while the file is open, and go to the device with one copy.

    with GgufFile(path) as g:
        n_expert = g.u64("gpt-oss.expert_count")
        bank = load_moe_block(ctx, g, block=0)      # device buffers, as stored
        layer = MoeLayer(ctx, bank.n_embd, bank.n_ff, bank.n_expert, k, gating, act, bank.wtype)
        layer.pack(bank.gate, bank.up, bank.down)
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from .kernels import Context, DeviceBuffer

# per-block tensor suffixes, as llama.cpp's GGUF writer spells them (tensors.rs names)
FFN_GATE_INP = "ffn_gate_inp.weight"
FFN_GATE_INP_BIAS = "ffn_gate_inp.bias"
FFN_GATE_EXPS = "ffn_gate_exps.weight"
FFN_UP_EXPS = "ffn_up_exps.weight"
FFN_DOWN_EXPS = "ffn_down_exps.weight"


class GgufError(RuntimeError):
    """The file could not be opened or is not a well-formed GGUF file."""


@dataclass(frozen=True)
class TensorInfo:
    name: str
    dims: tuple[int, ...]  # fastest-varying first, as stored
    type_id: int
    offset: int            # of the first byte, from the start of the file
    nbytes: int
    ptr: int               # address in the mapping

    def bytes(self) -> np.ndarray:
        """The tensor's bytes: a uint8 view of the mapping (valid while the file is open)."""
        if self.nbytes == 0:
            return np.empty(0, np.uint8)
        buf = (C.c_uint8 * self.nbytes).from_address(self.ptr)
        return np.frombuffer(buf, np.uint8)


class GgufFile:
    def __init__(self, path: str):
        self.lib = _lib.load()
        self.path = path
        self.h = self.lib.moearc_x_gguf_open(path.encode())
        if not self.h:
            raise GgufError(self.lib.moearc_x_gguf_last_error().decode(errors="replace"))

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.moearc_x_gguf_close(self.h)
            self.h = None

    def __enter__(self) -> "GgufFile":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self) -> None:
        self.close()

    @property
    def version(self) -> int:
        return self.lib.moearc_x_gguf_version(self.h)

    @property
    def alignment(self) -> int:
        return self.lib.moearc_x_gguf_alignment(self.h)

    @property
    def n_tensors(self) -> int:
        return self.lib.moearc_x_gguf_n_tensors(self.h)

    def _error(self) -> str:
        return self.lib.moearc_x_gguf_last_error().decode(errors="replace")

    def u64(self, key: str, default=None):
        v = C.c_ulonglong()
        if self.lib.moearc_x_gguf_key_u64(self.h, key.encode(), C.byref(v)) != 0:
            if default is not None:
                return default
            raise KeyError(self._error())
        return v.value

    def f64(self, key: str, default=None):
        v = C.c_double()
        if self.lib.moearc_x_gguf_key_f64(self.h, key.encode(), C.byref(v)) != 0:
            if default is not None:
                return default
            raise KeyError(self._error())
        return v.value

    def str(self, key: str, default=None):
        v = C.c_char_p()
        if self.lib.moearc_x_gguf_key_str(self.h, key.encode(), C.byref(v)) != 0:
            if default is not None:
                return default
            raise KeyError(self._error())
        return v.value.decode(errors="replace")

    @staticmethod
    def _info(name: str, t: _lib.GgufTensor) -> TensorInfo:
        return TensorInfo(name, tuple(int(t.dims[d]) for d in range(t.n_dims)), int(t.type_id), int(t.offset),
                          int(t.nbytes), int(t.data or 0))

    def has(self, name: str) -> bool:
        t = _lib.GgufTensor()
        return self.lib.moearc_x_gguf_find(self.h, name.encode(), C.byref(t)) == 0

    def tensor(self, name: str) -> TensorInfo:
        t = _lib.GgufTensor()
        if self.lib.moearc_x_gguf_find(self.h, name.encode(), C.byref(t)) != 0:
            raise KeyError(self._error())
        return self._info(name, t)

    def tensors(self) -> list[TensorInfo]:
        out = []
        for i in range(self.n_tensors):
            t = _lib.GgufTensor()
            nm = C.c_char_p()
            if self.lib.moearc_x_gguf_tensor_at(self.h, i, C.byref(t), C.byref(nm)) != 0:
                raise GgufError(self._error())
            out.append(self._info(nm.value.decode(errors="replace"), t))
        return out

    def slice_last(self, name: str, index: int) -> TensorInfo:
        """Slice `index` along the last dimension: one expert of a stacked expert bank
        (tensors.rs:237-289); ValueError when the slices do not tile the tensor exactly."""
        t = _lib.GgufTensor()
        if self.lib.moearc_x_gguf_slice_last(self.h, name.encode(), index, C.byref(t)) != 0:
            raise ValueError(self._error())
        return self._info(f"{name}[{index}]", t)

    def block_tensor(self, block: int, suffix: str) -> TensorInfo:
        return self.tensor(f"blk.{block}.{suffix}")


EXPERT_BANKS = (FFN_GATE_EXPS, FFN_UP_EXPS, FFN_DOWN_EXPS)


@dataclass(frozen=True)
class MoeLayout:
    """What sizing an expert pool or residency cache needs to know about a model file (the
    expert half of the reference's ModelInfo, crates/moearc-model/src/lib.rs:142-230)."""
    architecture: str
    block_count: int
    moe_blocks: tuple[int, ...]   # blocks that hold stacked expert banks
    n_expert: int
    n_expert_used: int
    per_expert_bytes: int         # gate + up + down of one expert (the largest, if they differ)
    per_expert_uniform: bool      # every MoE block's experts are the same size
    expert_bytes: int             # every stacked expert bank
    dense_bytes: int              # every other tensor


def moe_layout(g: GgufFile) -> MoeLayout:
    """The expert geometry of a MoE model file: which blocks hold stacked banks, one expert's
    bytes per block (each bank sliced exactly, tensors.rs:237-289), and the split of the file's
    weights into expert and dense bytes. ValueError for a file without experts."""
    arch = g.str("general.architecture")
    n_expert = g.u64(f"{arch}.expert_count", default=0)
    if not n_expert:
        raise ValueError(f"{g.path}: a {arch} file with no {arch}.expert_count is not a mixture of experts")
    used = g.u64(f"{arch}.expert_used_count")
    blocks = g.u64(f"{arch}.block_count")
    expert_bytes = dense_bytes = 0
    per_block: dict[int, int] = {}
    for t in g.tensors():
        parts = t.name.split(".", 2)
        if len(parts) == 3 and parts[0] == "blk" and parts[1].isdigit() and parts[2] in EXPERT_BANKS:
            if t.dims[-1] != n_expert:
                raise ValueError(f"{t.name} stacks {t.dims[-1]} experts, the file says {n_expert}")
            expert_bytes += t.nbytes
            per_block[int(parts[1])] = per_block.get(int(parts[1]), 0) + g.slice_last(t.name, 0).nbytes
        else:
            dense_bytes += t.nbytes
    sizes = set(per_block.values())
    return MoeLayout(arch, blocks, tuple(sorted(per_block)), n_expert, used, max(sizes, default=0),
                     len(sizes) <= 1, expert_bytes, dense_bytes)


@dataclass
class MoeBlockBanks:
    """A MoE block's tensors on the device, as stored in the file."""
    n_embd: int
    n_ff: int
    n_expert: int
    wtype: int
    gate: DeviceBuffer
    up: DeviceBuffer
    down: DeviceBuffer
    router: DeviceBuffer               # f32 [n_expert][n_embd]
    router_bias: DeviceBuffer | None   # f32 [n_expert] or None


def load_moe_block(ctx: Context, g: GgufFile, block: int) -> MoeBlockBanks:
    """Upload block `block`'s router and stacked expert banks (blk.N.ffn_{gate,up,down}_exps
    and ffn_gate_inp) to the device, one copy each straight from the mapping, after checking
    that their shapes agree: gate and up [n_embd, n_ff, n_expert], down [n_ff, n_embd,
    n_expert], one quantisation for the three, the router f32 [n_embd, n_expert]."""
    gate = g.block_tensor(block, FFN_GATE_EXPS)
    up = g.block_tensor(block, FFN_UP_EXPS)
    down = g.block_tensor(block, FFN_DOWN_EXPS)
    router = g.block_tensor(block, FFN_GATE_INP)
    if len(gate.dims) != 3 or gate.dims != up.dims:
        raise ValueError(f"block {block}: gate {gate.dims} and up {up.dims} banks differ or are not rank 3")
    H, I, E = gate.dims
    if down.dims != (I, H, E):
        raise ValueError(f"block {block}: down bank {down.dims} does not match gate {gate.dims}")
    if not (gate.type_id == up.type_id == down.type_id):
        raise ValueError(f"block {block}: experts mix types {gate.type_id}/{up.type_id}/{down.type_id}")
    if router.type_id != 0 or router.dims != (H, E):
        raise ValueError(f"block {block}: router {router.dims} type {router.type_id} is not f32 [{H}, {E}]")
    for t in (gate, up, down):
        for e in (0, E - 1):
            g.slice_last(t.name, e)  # the experts tile the bank exactly (raises otherwise)

    def up_load(t: TensorInfo) -> DeviceBuffer:
        b = ctx.alloc(t.nbytes)
        ctx._finish(ctx.lib.moearc_copy_h2d(ctx.raw, b.ptr, t.ptr, t.nbytes), "gguf upload")
        return b

    bias = None
    name = f"blk.{block}.{FFN_GATE_INP_BIAS}"
    if g.has(name):
        bt = g.tensor(name)
        if bt.type_id != 0 or bt.dims != (E,):
            raise ValueError(f"block {block}: router bias {bt.dims} type {bt.type_id} is not f32 [{E}]")
        bias = up_load(bt)
    return MoeBlockBanks(H, I, E, gate.type_id, up_load(gate), up_load(up), up_load(down), up_load(router), bias)
