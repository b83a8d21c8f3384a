"""experts.bin: the packed routed-expert records on disk, and their way into HBM.

The file format is the reference's (tools/repack_experts.py:1-8, manifest fields :233-252), kept byte for byte so
that a file packed by the reference loads here unchanged and a file written here loads there:

* ``<stem>.bin``: one record per (layer, expert) at byte ``(layer * experts + e) * record_bytes``; a record is the
  nine pieces gate/up/down x weight/scales/biases back to back (``records.RecordLayout`` gives their offsets).
* ``<stem>.manifest.json``: ``version`` 1, ``layout`` "slotstream-pool-layer-expert-piece-v1", ``layers``,
  ``experts``, ``pieces`` (bytes per piece), ``piece_names``, ``piece_offsets``, ``record_bytes``, ``alignment``
  4096 (a layer's bytes are a multiple of it), ``layer_sha256`` (SHA-256 of each layer's bytes), ``total_bytes``,
  and provenance fields (``model_identity``, ``source``, ``repacker``, ``stamp``) that the loader does not need.

On B200 the whole file fits in HBM: the reference model's 48 layers x 512 records of 2,764,800 bytes are 68 GB of
the 180 GB, so ``to_device`` loads every record once (file -> two pinned bounce buffers -> HBM, the read of one
chunk overlapping the copy of the previous one) and ``resident_tables`` gives the decode kernels their identity
map. The gate/up pieces stay in the reference order (no N-interleave): the kernels read gate and up rows of the same
output columns from their two pieces directly, so an interleaved copy would change no load the kernels issue.

Writing (``write_experts_bin``) follows the reference's crash-safe protocol: data goes to ``<stem>.bin.tmp``, a
layer's SHA-256 is recorded in ``<stem>.progress.json`` only after the layer is written and fsynced, a rerun skips
the layers the progress file holds, and the tmp file is renamed and the manifest written only when every layer has
its SHA. It packs records that a caller supplies per layer (a checkpoint reader, the synthetic generator); reading
the MLX checkpoint itself is the reference's job and stays there.
"""
import hashlib
import json
import os
from pathlib import Path

import numpy as np
import torch

from .records import EXPERTS_PER_LAYER, MAP_LAYERS, RecordLayout

LAYOUT_NAME = "slotstream-pool-layer-expert-piece-v1"
FORMAT_VERSION = 1
ALIGNMENT = 4096
PIECE_NAMES = tuple(f"{p}.{k}" for p in ("gate_proj", "up_proj", "down_proj") for k in ("weight", "scales", "biases"))


class ManifestError(ValueError):
    """The manifest or the file beside it does not describe a usable experts.bin."""


def layout_of(pieces, hidden: int) -> RecordLayout:
    """The record layout whose nine piece sizes are ``pieces``, given the model's hidden size (the manifest holds
    byte counts, not shapes): inter from the gate weight (inter * hidden / 2 bytes), the group size from its scales
    (inter * hidden / gs bf16 values)."""
    p = [int(v) for v in pieces]
    if len(p) != 9 or hidden <= 0:
        raise ManifestError("need nine piece sizes and a positive hidden size")
    inter, rem = divmod(2 * p[0], hidden)
    if rem or inter <= 0 or p[1] <= 0 or (inter * hidden * 2) % p[1]:
        raise ManifestError(f"piece sizes {p[:3]} do not fit hidden={hidden}")
    try:
        lay = RecordLayout(hidden, inter, inter * hidden * 2 // p[1])
    except ValueError as e:
        raise ManifestError(str(e)) from None
    want = [lay.w_bytes, lay.sb_bytes, lay.sb_bytes] * 3
    if p != want:
        raise ManifestError(f"piece sizes {p} are not those of {lay} ({want})")
    return lay


def _check_manifest(man: dict, file_bytes: int):
    need = ("version", "layout", "layers", "experts", "pieces", "piece_names", "piece_offsets", "record_bytes",
            "alignment", "layer_sha256", "total_bytes")
    missing = [k for k in need if k not in man]
    if missing:
        raise ManifestError(f"manifest lacks {missing}")
    if man["version"] != FORMAT_VERSION or man["layout"] != LAYOUT_NAME:
        raise ManifestError(f"unknown format {man['layout']!r} version {man['version']}")
    if list(man["piece_names"]) != list(PIECE_NAMES):
        raise ManifestError(f"piece order {man['piece_names']} is not {list(PIECE_NAMES)}")
    pieces, offs, rb = [int(v) for v in man["pieces"]], [int(v) for v in man["piece_offsets"]], int(man["record_bytes"])
    if len(pieces) != 9 or sum(pieces) != rb or offs != [int(v) for v in np.cumsum([0] + pieces[:-1])]:
        raise ManifestError("piece sizes, offsets and record_bytes disagree")
    nl, ne = int(man["layers"]), int(man["experts"])
    if nl <= 0 or ne <= 0 or len(man["layer_sha256"]) != nl:
        raise ManifestError("layers / experts / layer_sha256 disagree")
    if (ne * rb) % int(man["alignment"]):
        raise ManifestError(f"a layer ({ne} x {rb} bytes) is not a multiple of {man['alignment']}")
    if int(man["total_bytes"]) != nl * ne * rb or file_bytes != nl * ne * rb:
        raise ManifestError(f"file holds {file_bytes} bytes; the manifest describes {nl} x {ne} x {rb}")


class ExpertsFile:
    """A packed experts file opened read-only (memory-mapped): records, pieces and layers as numpy views."""

    def __init__(self, packed_dir, hidden: int = None, *, stem: str = "experts", verify: bool = False):
        d = Path(packed_dir)
        self.path = d / f"{stem}.bin"
        self.manifest = json.loads((d / f"{stem}.manifest.json").read_text())
        _check_manifest(self.manifest, os.stat(self.path).st_size)
        m = self.manifest
        self.layers, self.experts, self.record_bytes = int(m["layers"]), int(m["experts"]), int(m["record_bytes"])
        self.piece_offsets = tuple(int(v) for v in m["piece_offsets"])
        self.piece_sizes = tuple(int(v) for v in m["pieces"])
        self.layout = layout_of(self.piece_sizes, hidden) if hidden is not None else None
        self.data = np.memmap(self.path, dtype=np.uint8, mode="r",
                              shape=(self.layers, self.experts, self.record_bytes))
        if verify:
            bad = self.verify()
            if bad:
                raise ManifestError(f"layers {bad[:8]} do not match their SHA-256")

    def record(self, layer: int, e: int) -> np.ndarray:
        return self.data[layer, e]

    def piece(self, layer: int, e: int, j: int) -> np.ndarray:
        o = self.piece_offsets[j]
        return self.data[layer, e, o:o + self.piece_sizes[j]]

    def layer_records(self, layer: int) -> np.ndarray:
        return self.data[layer]

    def verify(self, layers=None):
        """Layers whose bytes do not hash to the manifest's layer_sha256 (empty when the file is intact)."""
        bad = []
        for L in (range(self.layers) if layers is None else layers):
            if hashlib.sha256(self.data[L]).hexdigest() != self.manifest["layer_sha256"][L]:
                bad.append(int(L))
        return bad

    def to_pinned(self, layers=None) -> torch.Tensor:
        """uint8 [n_layers, experts, record_bytes] in pinned host memory (the host side of a slot pool or a sweep)."""
        ls = list(range(self.layers)) if layers is None else list(layers)
        out = torch.empty((len(ls), self.experts, self.record_bytes), dtype=torch.uint8).pin_memory()
        for i, L in enumerate(ls):
            out[i].numpy()[...] = self.data[L]
        return out

    def to_device(self, layers=None, device="cuda", chunk_bytes: int = 256 << 20) -> torch.Tensor:
        """uint8 [n_layers, experts, record_bytes] in HBM. The file is read into two pinned bounce buffers in
        turn; each buffer's copy to the device runs while the next chunk is read into the other one."""
        ls = list(range(self.layers)) if layers is None else list(layers)
        lb = self.experts * self.record_bytes
        out = torch.empty((len(ls), self.experts, self.record_bytes), dtype=torch.uint8, device=device)
        flat = out.view(-1)
        chunk = max(ALIGNMENT, min(int(chunk_bytes), lb) // ALIGNMENT * ALIGNMENT)
        bounce = [torch.empty(chunk, dtype=torch.uint8).pin_memory() for _ in range(2)]
        done = [None, None]
        stream = torch.cuda.Stream(device=device)
        n = 0
        with torch.cuda.stream(stream):
            for i, L in enumerate(ls):
                src = self.data[L].reshape(-1)
                for a in range(0, lb, chunk):
                    b = min(lb, a + chunk)
                    s = n % 2
                    if done[s] is not None:
                        done[s].synchronize()             # the copy that last read this buffer has finished
                    bounce[s][:b - a].numpy()[...] = src[a:b]
                    flat[i * lb + a:i * lb + b].copy_(bounce[s][:b - a], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(stream)
                    done[s] = ev
                    n += 1
        stream.synchronize()
        return out

    def resident_tables(self, records: torch.Tensor, first_layer: int = 0):
        """(map_t int32 [MAP_LAYERS * 512], slot_ptr_t int64 [n]) for decode kernels reading ``records`` (a
        ``to_device`` result of consecutive layers from ``first_layer``): expert e of layer L sits in slot
        (L - first_layer) * experts + e."""
        if self.experts != EXPERTS_PER_LAYER:
            raise ManifestError(f"decode tables index 512 experts per layer, the file has {self.experts}")
        nl = records.shape[0]
        if first_layer < 0 or first_layer + nl > MAP_LAYERS:
            raise ValueError("layers outside the decode map")
        dev = records.device
        n = nl * self.experts
        map_t = torch.full((MAP_LAYERS * self.experts,), -1, dtype=torch.int32, device=dev)
        lo = first_layer * self.experts
        map_t[lo:lo + n] = torch.arange(n, dtype=torch.int32, device=dev)
        slot_ptr = records.data_ptr() + torch.arange(n, dtype=torch.int64, device=dev) * self.record_bytes
        return map_t, slot_ptr


def _atomic_json(path: Path, obj):
    part = Path(str(path) + ".part")
    with open(part, "w") as f:
        json.dump(obj, f, indent=1)
        f.flush()
        os.fsync(f.fileno())
    os.replace(part, path)


def write_experts_bin(out_dir, layers: int, experts: int, piece_sizes, layer_fn, *, stem: str = "experts",
                      model_identity: str = None, source=None):
    """Pack ``layers`` layers into ``<stem>.bin`` + manifest. ``layer_fn(L)`` returns uint8 [experts, record_bytes]
    (the nine pieces of each expert back to back). Resumable: layers already in ``<stem>.progress.json`` beside an
    existing ``<stem>.bin.tmp`` of the right size are kept. Returns a summary with the layers written by this call."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    sizes = [int(v) for v in piece_sizes]
    if len(sizes) != 9:
        raise ValueError("need the nine piece sizes")
    rb = sum(sizes)
    lb = experts * rb
    if lb % ALIGNMENT:
        raise ValueError(f"a layer ({experts} x {rb} bytes) must be a multiple of {ALIGNMENT} bytes")
    final, tmp = out / f"{stem}.bin", out / f"{stem}.bin.tmp"
    prog_path, man_path = out / f"{stem}.progress.json", out / f"{stem}.manifest.json"
    total = layers * lb
    if final.exists() and man_path.exists() and not tmp.exists():
        return {"status": "already done", "path": str(final)}
    fd = os.open(tmp, os.O_RDWR | os.O_CREAT, 0o644)
    try:
        fresh = os.fstat(fd).st_size != total
        if fresh:
            os.ftruncate(fd, 0)
            os.ftruncate(fd, total)
        progress = {}
        if not fresh and prog_path.exists():
            progress = {int(k): v for k, v in json.loads(prog_path.read_text()).items()}
        written = []
        for L in range(layers):
            if L in progress:
                continue
            arr = np.ascontiguousarray(layer_fn(L), dtype=np.uint8)
            if arr.shape != (experts, rb):
                raise ValueError(f"layer {L}: want uint8 [{experts}, {rb}], got {arr.shape}")
            mv = memoryview(arr).cast("B")
            done = 0
            while done < lb:
                done += os.pwrite(fd, mv[done:], L * lb + done)
            os.fsync(fd)
            progress[L] = hashlib.sha256(mv).hexdigest()
            _atomic_json(prog_path, {str(k): v for k, v in sorted(progress.items())})
            written.append(L)
    finally:
        os.close(fd)
    os.replace(tmp, final)
    dfd = os.open(out, os.O_RDONLY)
    try:
        os.fsync(dfd)
    finally:
        os.close(dfd)
    st = os.stat(final)
    manifest = {
        "version": FORMAT_VERSION, "layout": LAYOUT_NAME, "model_identity": model_identity, "layers": layers,
        "experts": experts, "pieces": sizes, "piece_names": list(PIECE_NAMES),
        "piece_offsets": [int(v) for v in np.cumsum([0] + sizes[:-1])], "record_bytes": rb, "alignment": ALIGNMENT,
        "layer_sha256": [progress[L] for L in range(layers)],
        "source": source or {"repo": "unknown", "revision": "unknown"},
        "repacker": {"path": "slotstream_b200/experts_file.py"},
        "stamp": {"dev": st.st_dev, "ino": st.st_ino, "size": st.st_size, "mtime_ns": st.st_mtime_ns,
                  "ctime_ns": st.st_ctime_ns},
        "total_bytes": total,
    }
    _atomic_json(man_path, manifest)
    return {"path": str(final), "layers": layers, "experts": experts, "record_bytes": rb, "total_bytes": total,
            "written_layers": written}
