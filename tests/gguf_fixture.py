"""GGUF byte builders for the reader and loader tests.

`Fixture` builds a container the way the reference's reader tests do
(bridge-gguf/tests/reader.rs:72-171): metadata records and tensor records
as given (offsets included, so malformed directories can be written), the
data section at the next multiple of the alignment, then the payload.

`write_hy3` writes a Hy3 GGUF set with MoE blocks in the reference schema
(bridge-model-hy3/src/schema.rs:200-258: exp_probs_b, ffn_gate_inp, stacked
ffn_{gate,up,down}_exps, ffn_{gate,up,down}_shexp) and the hy_v3.* keys that
resolve_config reads (config.rs:57-109), optionally split into numbered
shards with split.no / split.count / split.tensors.count.
"""

from __future__ import annotations

import pathlib
import struct

import numpy as np

import synth

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
GGML_F32 = 0


class Fixture:
    def __init__(self, version: int = 3, big: bool = False):
        self.version = version
        self.big = big
        self.metadata: list[bytes] = []
        self.tensors: list[bytes] = []
        self.payload = b""
        self.alignment = 32

    def _p(self, fmt: str, v) -> bytes:
        return struct.pack((">" if self.big else "<") + fmt, v)

    def u8(self, v):
        return self._p("B", v)

    def u16(self, v):
        return self._p("H", v)

    def i32(self, v):
        return self._p("i", v)

    def u32(self, v):
        return self._p("I", v)

    def u64(self, v):
        return self._p("Q", v)

    def f32(self, v):
        return self._p("f", v)

    def string(self, b: bytes) -> bytes:
        return self.u64(len(b)) + b

    def array(self, element_type: int, elements: bytes, count: int) -> bytes:
        return self.u32(element_type) + self.u64(count) + elements

    def meta(self, key: bytes, ty: int, value: bytes) -> "Fixture":
        self.metadata.append(self.string(key) + self.u32(ty) + value)
        return self

    def tensor(self, name: bytes, dims, ty: int, offset: int) -> "Fixture":
        rec = self.string(name) + self.u32(len(dims))
        for d in dims:
            rec += self.u64(d)
        self.tensors.append(rec + self.u32(ty) + self.u64(offset))
        return self

    def add_payload(self, b: bytes) -> "Fixture":
        self.payload += bytes(b)
        return self

    def bytes(self, tensor_count: int | None = None, metadata_count: int | None = None) -> bytes:
        out = (b"FUGG" if self.big else b"GGUF") + self.u32(self.version)
        out += self.u64(len(self.tensors) if tensor_count is None else tensor_count)
        out += self.u64(len(self.metadata) if metadata_count is None else metadata_count)
        for m in self.metadata:
            out += m
        for t in self.tensors:
            out += t
        pad = -len(out) % self.alignment
        return out + b"\0" * pad + self.payload


def _pad(n: int, a: int = 32) -> int:
    return (n + a - 1) // a * a


class Hy3Block:
    """One MoE block's host tensors, GGUF layout: router [E, H] f32 rows, bias
    [E], experts [(gate, up, down)] packed bytes, shared (gate, up, down)."""

    def __init__(self, rng, H, F, E, gty, uty, dty, sgty, suty, sdty):
        self.router = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
        self.bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
        self.types = (gty, uty, dty, sgty, suty, sdty)
        self.experts = [(synth.packed_np(rng, gty, H, F), synth.packed_np(rng, uty, H, F), synth.packed_np(rng, dty, F, H))
                        for _ in range(E)]
        self.shared = (synth.packed_np(rng, sgty, H, F), synth.packed_np(rng, suty, H, F), synth.packed_np(rng, sdty, F, H))

    def tensors(self, b: int, H: int, F: int, E: int):
        gty, uty, dty, sgty, suty, sdty = self.types
        p = f"blk.{b}."
        return [
            (p + "exp_probs_b", [E], GGML_F32, self.bias.tobytes()),
            (p + "ffn_gate_inp.weight", [H, E], GGML_F32, self.router.tobytes()),
            (p + "ffn_gate_exps.weight", [H, F, E], gty, b"".join(e[0].tobytes() for e in self.experts)),
            (p + "ffn_up_exps.weight", [H, F, E], uty, b"".join(e[1].tobytes() for e in self.experts)),
            (p + "ffn_down_exps.weight", [F, H, E], dty, b"".join(e[2].tobytes() for e in self.experts)),
            (p + "ffn_gate_shexp.weight", [H, F], sgty, self.shared[0].tobytes()),
            (p + "ffn_up_shexp.weight", [H, F], suty, self.shared[1].tobytes()),
            (p + "ffn_down_shexp.weight", [F, H], sdty, self.shared[2].tobytes()),
        ]


def hy3_metadata(fx: Fixture, H, F, E, k, blocks, scale=2.826, shared_ffn=None, arch=b"hy_v3") -> None:
    fx.meta(b"general.architecture", STRING, fx.string(arch))
    fx.meta(b"general.alignment", U32, fx.u32(fx.alignment))
    for key, v in [("block_count", blocks), ("embedding_length", H), ("expert_feed_forward_length", F),
                   ("expert_shared_feed_forward_length", F if shared_ffn is None else shared_ffn),
                   ("expert_count", E), ("expert_used_count", k)]:
        fx.meta(f"hy_v3.{key}".encode(), U32, fx.u32(v))
    fx.meta(b"hy_v3.expert_weights_scale", F32, fx.f32(scale))
    tokens = b"".join(fx.string(t) for t in (b"<s>", b"</s>", b"hy"))
    fx.meta(b"tokenizer.ggml.tokens", ARRAY, fx.array(STRING, tokens, 3))


def write_hy3(directory, H, F, E, k, blocks: dict[int, Hy3Block], block_count=None, shards: int = 1,
              prefix: str = "hy3", scale: float = 2.826, extra_meta=None, alignment: int = 32) -> pathlib.Path:
    """Writes the set and returns the entry path (the first shard). Tensors are
    dealt to shards block by block, in block order."""
    directory = pathlib.Path(directory)
    block_count = max(blocks) + 1 if block_count is None else block_count
    entries = []
    for b in sorted(blocks):
        entries += blocks[b].tensors(b, H, F, E)
    per = [[] for _ in range(shards)]
    for i, b in enumerate(sorted(blocks)):
        per[i * shards // len(blocks)].extend(blocks[b].tensors(b, H, F, E))
    paths = []
    for s in range(shards):
        fx = Fixture()
        fx.alignment = alignment
        if s == 0:
            hy3_metadata(fx, H, F, E, k, block_count, scale)
            for key, ty, val in extra_meta or []:
                fx.meta(key, ty, val)
        if shards > 1:
            fx.meta(b"split.no", U16, fx.u16(s))
            fx.meta(b"split.count", U16, fx.u16(shards))
            fx.meta(b"split.tensors.count", I32, fx.i32(len(entries)))
        off = 0
        for name, dims, ty, payload in per[s]:
            fx.tensor(name.encode(), dims, ty, off)
            fx.add_payload(payload + b"\0" * (_pad(len(payload), alignment) - len(payload)))
            off += _pad(len(payload), alignment)
        name = f"{prefix}.gguf" if shards == 1 else f"{prefix}-{s + 1:05d}-of-{shards:05d}.gguf"
        path = directory / name
        path.write_bytes(fx.bytes())
        paths.append(path)
    return paths[0]
