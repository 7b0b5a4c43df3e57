"""GGUF files for the MoE block: the tensors' raw bytes as zero-copy views of the file's memory map, and the MoE
configuration from the metadata; plus a writer for synthetic files.

Follows the reference's ``GGUFFile`` (src/artlite/gguf_model.py:396-506): GGUF v2/v3, metadata key/value types
(:380-382), the ggml type table (:385-390), tensor data at ``align(end of infos, general.alignment)`` + offset, a
tensor as (rows, row_bytes) with the blocks along the row (dims[0] = cols). The MoE keys follow
``QwenConfig`` (src/artlite/model_config.py:853-898): ``{arch}.expert_count``, ``expert_used_count``,
``expert_feed_forward_length``, ``embedding_length``; the tensor names ``blk.L.ffn_{gate,up,down}_exps.weight`` and
``blk.L.ffn_gate_inp.weight`` (tests/moe/ref.py:27-40)."""

import math
import struct
from dataclasses import dataclass

import numpy as np

_KV_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
_KV_STRING, _KV_ARRAY = 8, 9
# ggml type id: (name, values per block, bytes per block)
GGML_TYPES = {0: ("F32", 1, 4), 1: ("F16", 1, 2), 2: ("Q4_0", 32, 18), 3: ("Q4_1", 32, 20), 8: ("Q8_0", 32, 34),
              10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110), 12: ("Q4_K", 256, 144), 13: ("Q5_K", 256, 176),
              14: ("Q6_K", 256, 210), 20: ("IQ4_NL", 32, 18), 23: ("IQ4_XS", 256, 136), 30: ("BF16", 1, 2)}
TYPE_IDS = {v[0]: k for k, v in GGML_TYPES.items()}


@dataclass
class RawTensor:
    name: str
    qtype: str
    rows: int
    cols: int
    raw: np.ndarray  # (rows, row_bytes) uint8 view of the mapped file


class GGUFFile:
    """A GGUF file parsed from its memory map: ``meta`` (scalars, strings, numeric arrays), ``tensor(name)`` a
    zero-copy RawTensor."""

    def __init__(self, path: str):
        self.path = path
        self.data = np.memmap(path, dtype=np.uint8, mode="r")
        buf = memoryview(self.data)
        if bytes(buf[:4]) != b"GGUF":
            raise ValueError(f"{path}: not a GGUF file")
        version, n_tensors, n_kv = struct.unpack_from("<IQQ", buf, 4)
        if version not in (2, 3):
            raise ValueError(f"{path}: GGUF version {version}")
        pos = 24
        self.meta: dict[str, object] = {}

        def string(pos: int) -> tuple[str, int]:
            n = int.from_bytes(buf[pos:pos + 8], "little")
            return bytes(buf[pos + 8:pos + 8 + n]).decode("utf-8", errors="replace"), pos + 8 + n

        for _ in range(n_kv):
            key, pos = string(pos)
            (vt,) = struct.unpack_from("<I", buf, pos)
            pos += 4
            if vt == _KV_STRING:
                self.meta[key], pos = string(pos)
            elif vt == _KV_ARRAY:
                et, count = struct.unpack_from("<IQ", buf, pos)
                pos += 12
                if et == _KV_STRING:
                    vals = []
                    for _ in range(count):
                        s, pos = string(pos)
                        vals.append(s)
                    self.meta[key] = vals
                else:
                    dt = np.dtype(_KV_SCALAR[et])
                    self.meta[key] = np.frombuffer(buf, dt, count, pos)
                    pos += count * dt.itemsize
            else:
                fmt = _KV_SCALAR[vt]
                (self.meta[key],) = struct.unpack_from(fmt, buf, pos)
                pos += struct.calcsize(fmt)
        self.arch = str(self.meta.get("general.architecture", ""))
        infos = []
        for _ in range(n_tensors):
            name, pos = string(pos)
            (nd,) = struct.unpack_from("<I", buf, pos)
            dims = struct.unpack_from(f"<{nd}Q", buf, pos + 4)
            ttype, off = struct.unpack_from("<IQ", buf, pos + 4 + 8 * nd)
            pos += 16 + 8 * nd
            infos.append((name, dims, ttype, off))
        align = int(self.meta.get("general.alignment", 32))
        base = -(-pos // align) * align
        self.tensor_info: dict[str, tuple[tuple[int, ...], str, int, int | None]] = {}
        for name, dims, ttype, off in infos:
            tname, per, nb = GGML_TYPES.get(ttype, (f"type{ttype}", 1, None))
            n = math.prod(dims)
            self.tensor_info[name] = (dims, tname, base + off, None if nb is None else n // per * nb)

    def arch_meta(self, key: str, default: object = None) -> object:
        return self.meta.get(f"{self.arch}.{key}", default)

    def __contains__(self, name: str) -> bool:
        return name in self.tensor_info

    def tensor(self, name: str) -> RawTensor:
        dims, qtype, off, nbytes = self.tensor_info[name]
        if nbytes is None:
            raise NotImplementedError(f"{name}: GGUF tensor type {qtype} is not supported")
        cols = dims[0]
        rows = math.prod(dims[1:]) if len(dims) > 1 else 1
        return RawTensor(name, qtype, rows, cols, self.data[off:off + nbytes].reshape(rows, -1))

    def moe_config(self) -> dict[str, int]:
        """The MoE block's shape from the metadata (model_config.py:853-898)."""
        return {"hidden": int(self.arch_meta("embedding_length")), "n_experts": int(self.arch_meta("expert_count")),
                "top_k": int(self.arch_meta("expert_used_count")),
                "expert_ffn": int(self.arch_meta("expert_feed_forward_length")),
                "n_layers": int(self.arch_meta("block_count"))}

    def moe_layer(self, layer: int) -> dict[str, RawTensor]:
        b = f"blk.{layer}."
        return {k: self.tensor(b + n) for k, n in (("gate", "ffn_gate_exps.weight"), ("up", "ffn_up_exps.weight"),
                                                   ("down", "ffn_down_exps.weight"), ("router", "ffn_gate_inp.weight"))}


def write_gguf(path: str, meta: dict[str, object], tensors: list[tuple[str, str, tuple[int, ...], np.ndarray]],
               alignment: int = 32) -> None:
    """A GGUF v3 file: ``meta`` values (int -> u32, float -> f32, str, bool), ``tensors`` (name, type name, dims with
    dims[0] the row length, raw bytes)."""

    def s(x: str) -> bytes:
        b = x.encode()
        return struct.pack("<Q", len(b)) + b

    kv = b""
    for k, v in meta.items():
        if isinstance(v, bool):
            kv += s(k) + struct.pack("<I?", 7, v)
        elif isinstance(v, int):
            kv += s(k) + struct.pack("<II", 4, v)
        elif isinstance(v, float):
            kv += s(k) + struct.pack("<If", 6, v)
        else:
            kv += s(k) + struct.pack("<I", _KV_STRING) + s(str(v))
    info, off, blobs = b"", 0, []
    for name, qtype, dims, raw in tensors:
        info += s(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
        info += struct.pack("<IQ", TYPE_IDS[qtype], off)
        blob = np.ascontiguousarray(raw).view(np.uint8).tobytes()
        blobs.append(blob)
        off += -(-len(blob) // alignment) * alignment
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(meta)) + kv + info
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (-(-len(head) // alignment) * alignment - len(head)))
        for blob in blobs:
            f.write(blob)
            f.write(b"\0" * (-(-len(blob) // alignment) * alignment - len(blob)))
