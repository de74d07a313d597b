"""The reference engine's ``.llmy`` checkpoint format: reader and writer.

Reference: llmy_cuda/tools/convert_checkpoint.py (writer) and
llmy_cuda/include/checkpoint.h (reader).  Little-endian throughout:

    offset  field
    0       magic "LLMY"
    4       version u32 (1)
    8       cfg_len u32
    12      config: cfg_len bytes of UTF-8 ``key=value`` lines, nested keys
            dotted (``csa.local_window=512``), lists comma-separated, booleans
            written as 1 / 0, keys sorted
    ...     n_tensors u32
    ...     index: n_tensors entries of 108 bytes (convert_checkpoint.py:47;
            the "96-byte" figure in both files' comments is stale):
              u32 name_len, char name[64] (NUL-padded), u32 dtype
              (0 f32, 1 f16, 2 bf16), u32 ndim (<= 4), u32 shape[4],
              u64 offset (from the data start), u64 nbytes
    data    starts at the first multiple of 4096 after the index; payloads
            back to back in index order (names sorted)

The converter stacks per-expert parameters (``...experts.<i>.<rest>``) into
``...experts.<rest>`` of shape [E, ...] (convert_checkpoint.py:265-297).
``read_llmy`` maps the file and returns zero-copy CPU tensors; ``write_llmy``
produces the converter's bytes for the same tensors and configuration.
"""
from __future__ import annotations

import mmap
import re
import struct
import warnings
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Mapping

import torch

MAGIC = b"LLMY"
VERSION = 1
INDEX_ENTRY = struct.Struct("<I64sII4IQQ")  # 108 bytes
DATA_ALIGN = 4096
_DTYPES = {0: torch.float32, 1: torch.float16, 2: torch.bfloat16}
_CODES = {v: k for k, v in _DTYPES.items()}
# top-level configuration keys the converter keeps (convert_checkpoint.py:73-79)
ALLOWED_KEYS = frozenset({
    "vocab_size", "d_model", "num_loops", "physical_blocks", "stem_blocks", "recurrent_blocks",
    "tail_blocks", "recurrent_layout", "max_position_embeddings", "mhc", "gdn", "moe", "mla",
    "router", "csa", "hca", "dense_ffn", "loop_attnres", "adaptive_loops",
})
_EXPERT_RE = re.compile(r"^(?P<prefix>.+\.(?:experts|shared))\.(?P<idx>\d+)\.(?P<rest>.+)$")


# ---------------------------------------------------------------- config text
def _fmt(v: Any) -> str:
    if isinstance(v, bool):
        return "1" if v else "0"
    if isinstance(v, (int, float)):
        return repr(v)
    if isinstance(v, str):
        return v
    if isinstance(v, (list, tuple)):
        return ",".join(str(x) for x in v)
    return str(v)


def _flatten(prefix: str, value: Any, out: dict[str, str]) -> None:
    if isinstance(value, dict):
        for k, v in value.items():
            _flatten(f"{prefix}.{k}" if prefix else k, v, out)
    else:
        out[prefix] = _fmt(value)


def flatten_config(cfg: Mapping[str, Any]) -> str:
    """The configuration text the converter embeds (convert_checkpoint.py:103-119):
    a ``{"model": {...}}`` wrapper is unwrapped, only ALLOWED_KEYS are kept."""
    if isinstance(cfg.get("model"), dict):
        cfg = cfg["model"]
    flat: dict[str, str] = {}
    for k, v in cfg.items():
        if k in ALLOWED_KEYS and isinstance(v, (dict, list, tuple, str, int, float, bool)):
            _flatten(k, v, flat)
    return "".join(f"{k}={flat[k]}\n" for k in sorted(flat))


def _scalar(text: str) -> Any:
    for conv in (int, float):
        try:
            return conv(text)
        except ValueError:
            pass
    return text


def parse_config(text: str) -> dict[str, Any]:
    """Nested mapping from the ``key=value`` text.  Values become int / float
    when they parse as such (booleans were written as 1 / 0), comma-separated
    values lists; ``recurrent_layout`` is always a list."""
    out: dict[str, Any] = {}
    for line in text.splitlines():
        if not line.strip():
            continue
        key, _, val = line.partition("=")
        value: Any = [_scalar(x) for x in val.split(",")] if "," in val else _scalar(val)
        if key == "recurrent_layout" and not isinstance(value, list):
            value = [value]
        node = out
        parts = key.split(".")
        for p in parts[:-1]:
            node = node.setdefault(p, {})
        node[parts[-1]] = value
    return out


# -------------------------------------------------------------------- tensors
def stack_experts(named: Mapping[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """``...experts.<i>.<rest>`` entries stacked into ``...experts.<rest>``
    [E, ...] in expert order; other entries unchanged."""
    groups: dict[tuple[str, str], list[tuple[int, torch.Tensor]]] = {}
    out: dict[str, torch.Tensor] = {}
    for name, t in named.items():
        m = _EXPERT_RE.match(name)
        if m is None:
            out[name] = t
        else:
            groups.setdefault((m["prefix"], m["rest"]), []).append((int(m["idx"]), t))
    for (prefix, rest), items in groups.items():
        items.sort(key=lambda kv: kv[0])
        if any(t.shape != items[0][1].shape for _, t in items):
            raise ValueError(f"expert shapes differ under {prefix}.{rest}")
        out[f"{prefix}.{rest}"] = torch.stack([t for _, t in items]).contiguous()
    return out


@dataclass
class LlmyFile:
    """A mapped ``.llmy`` file: configuration text and zero-copy tensors (in
    index order).  Keep the object alive while the tensors are used."""
    path: Path
    version: int
    config_text: str
    tensors: dict[str, torch.Tensor]
    _map: mmap.mmap | None = None

    @property
    def config(self) -> dict[str, Any]:
        return parse_config(self.config_text)

    def close(self) -> None:
        """Drop the tensors and unmap (left to the garbage collector while a
        caller still holds one of the tensors)."""
        self.tensors = {}
        if self._map is not None:
            try:
                self._map.close()
            except BufferError:
                pass
            self._map = None


def read_llmy(path: str | Path) -> LlmyFile:
    """Map and parse a ``.llmy`` file (llmy_cuda/include/checkpoint.h)."""
    path = Path(path)
    with path.open("rb") as f:
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
    try:
        if mm[:4] != MAGIC:
            raise ValueError(f"{path}: not an .llmy file")
        version, cfg_len = struct.unpack_from("<II", mm, 4)
        if version != VERSION:
            raise ValueError(f"{path}: unsupported version {version}")
        config_text = bytes(mm[12:12 + cfg_len]).decode("utf-8")
        pos = 12 + cfg_len
        (n,) = struct.unpack_from("<I", mm, pos)
        pos += 4
        index_end = pos + n * INDEX_ENTRY.size
        if index_end > len(mm):
            raise ValueError(f"{path}: index runs past the end of the file")
        data_start = index_end + (DATA_ALIGN - index_end % DATA_ALIGN) % DATA_ALIGN
        buf = memoryview(mm)
        tensors: dict[str, torch.Tensor] = {}
        for i in range(n):
            name_len, name, code, ndim, s0, s1, s2, s3, off, nbytes = INDEX_ENTRY.unpack_from(
                mm, pos + i * INDEX_ENTRY.size)
            if code not in _DTYPES or ndim > 4 or name_len > 63:
                raise ValueError(f"{path}: bad index entry {i}")
            shape = [s0, s1, s2, s3][:ndim]
            dtype = _DTYPES[code]
            start = data_start + off
            if start + nbytes > len(mm):
                raise ValueError(f"{path}: tensor {i} runs past the end of the file")
            if nbytes:
                with warnings.catch_warnings():  # the mapping is read-only by design
                    warnings.simplefilter("ignore", UserWarning)
                    raw = torch.frombuffer(buf[start:start + nbytes], dtype=torch.uint8)
            else:
                raw = torch.empty(0, dtype=torch.uint8)
            t = raw.view(dtype).reshape(shape)
            tensors[name[:name_len].decode("utf-8")] = t
    except Exception:
        tensors = {}
        try:
            mm.close()
        except BufferError:  # views of the mapping still alive: the collector unmaps it
            pass
        raise
    return LlmyFile(path, version, config_text, tensors, mm)


def write_llmy(path: str | Path, config: Mapping[str, Any] | str,
               tensors: Mapping[str, torch.Tensor]) -> None:
    """Write ``tensors`` (stacked with stack_experts, sorted by name) and the
    configuration (a mapping, flattened like the converter, or ready text)."""
    named = stack_experts({k.replace("_orig_mod.", ""): v.detach().contiguous().cpu()
                           for k, v in tensors.items()})
    items = sorted(named.items())
    text = config if isinstance(config, str) else flatten_config(config)
    cfg_b = text.encode("utf-8")
    with Path(path).open("wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<II", VERSION, len(cfg_b)))
        f.write(cfg_b)
        f.write(struct.pack("<I", len(items)))
        index_start = f.tell()
        f.write(b"\0" * (INDEX_ENTRY.size * len(items)))
        end = f.tell()
        f.write(b"\0" * ((DATA_ALIGN - end % DATA_ALIGN) % DATA_ALIGN))
        data_start = f.tell()
        entries = []
        for name, t in items:
            if t.dtype not in _CODES:
                raise ValueError(f"unsupported dtype {t.dtype} for {name}")
            if t.dim() > 4:
                raise ValueError(f"tensor {name} has {t.dim()} dims (max 4)")
            name_b = name.encode("utf-8")
            if len(name_b) > 63:
                raise ValueError(f"tensor name too long: {name}")
            blob = t.reshape(-1).view(torch.uint8).numpy().tobytes() if t.numel() else b""
            entries.append(INDEX_ENTRY.pack(len(name_b), name_b.ljust(64, b"\0"), _CODES[t.dtype],
                                            t.dim(), *(list(t.shape) + [0] * (4 - t.dim())),
                                            f.tell() - data_start, len(blob)))
            f.write(blob)
        f.seek(index_start)
        for e in entries:
            f.write(e)


# ------------------------------------------------------------------- converter
def convert_checkpoint(src: str | Path, dst: str | Path, *, keep_fp32: bool = False,
                       strict: bool = False) -> int:
    """The converter tool (llmy_cuda/tools/convert_checkpoint.py:122-222): a
    training checkpoint ``{"model": state_dict, "config": mapping}`` (or a bare
    state dict with a "config" entry) to ``.llmy``.  Non-tensor entries are
    skipped; keep_fp32 stores every tensor as float32; strict fails on any
    tensor that is not float32.  Returns the process exit status (0, or 1 with a
    message on stderr) at the same points as the tool; the messages are this
    project's own."""
    import sys
    src, dst = Path(src), Path(dst)
    if not src.is_file():
        print(f"llmy convert: cannot read {src}: no such file", file=sys.stderr)
        return 1
    ckpt = torch.load(src, map_location="cpu", weights_only=False)
    if not isinstance(ckpt, dict):
        print(f"llmy convert: {src} holds a {type(ckpt).__name__}, not a mapping", file=sys.stderr)
        return 1
    cfg = ckpt.get("config")
    if cfg is None:
        print(f"llmy convert: {src} carries no 'config' entry", file=sys.stderr)
        return 1
    if not isinstance(cfg, dict):
        print(f"llmy convert: the 'config' entry is a {type(cfg).__name__}; a mapping is required",
              file=sys.stderr)
        return 1
    state = ckpt.get("model", ckpt)
    if not isinstance(state, dict):
        print("llmy convert: the weights ('model' entry) are not a mapping", file=sys.stderr)
        return 1
    tensors: dict[str, torch.Tensor] = {}
    for name, t in state.items():
        if not isinstance(t, torch.Tensor):
            continue
        t = t.float() if keep_fp32 else t
        if strict and t.dtype != torch.float32:
            print(f"llmy convert: --strict: {name.replace('_orig_mod.', '')} has dtype {t.dtype}, "
                  "not float32", file=sys.stderr)
            return 1
        tensors[name] = t
    write_llmy(dst, cfg, tensors)
    return 0


def _main(argv: list[str] | None = None) -> int:
    import argparse
    ap = argparse.ArgumentParser(prog="python -m hybrid_llm_b200.llmy_format",
                                 description="Write a .llmy file from a training checkpoint, or print a "
                                             ".llmy file's configuration and tensor table.")
    sub = ap.add_subparsers(dest="cmd", required=True)
    cv = sub.add_parser("convert", help="pack a .pt training checkpoint into a .llmy file")
    cv.add_argument("input", type=Path)
    cv.add_argument("output", type=Path)
    cv.add_argument("--keep-fp32", action="store_true",
                    help="widen every tensor to float32 (otherwise each keeps its dtype)")
    cv.add_argument("--strict", action="store_true",
                    help="exit with status 1 if a tensor would be stored in a dtype other "
                         "than float32")
    ls = sub.add_parser("info", help="show a .llmy file's configuration text and its tensors "
                         "(name, dtype, shape)")
    ls.add_argument("file", type=Path)
    args = ap.parse_args(argv)
    if args.cmd == "convert":
        return convert_checkpoint(args.input, args.output, keep_fp32=args.keep_fp32,
                                  strict=args.strict)
    f = read_llmy(args.file)
    try:
        print(f.config_text, end="")
        for name, t in f.tensors.items():
            print(f"{name}\t{str(t.dtype).replace('torch.', '')}\t{list(t.shape)}")
    finally:
        f.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(_main())
