"""experts.bin loading and writing (slotstream_b200.experts_file) against a file the reference's own repacker
produced (tools/repack_experts.py on tests/t0/synth_ckpt.py's checkpoint, fixture experts_bin/ made by
make_golden.py), plus the crash-safe resume and the manifest checks (tests/t0/test_repack_experts.py:31-77)."""
import hashlib
import json
import shutil

import numpy as np
import pytest

from conftest import GOLDEN
from slotstream_b200 import synth
from slotstream_b200.experts_file import (PIECE_NAMES, ExpertsFile, ManifestError, layout_of,
                                          write_experts_bin)
from slotstream_b200.records import RecordLayout

REF = GOLDEN / "experts_bin"
FORMAT_KEYS = ("version", "layout", "layers", "experts", "pieces", "piece_names", "piece_offsets", "record_bytes",
               "alignment", "layer_sha256", "total_bytes")


def test_reference_packed_file_loads_with_its_pieces_in_place():
    ef = ExpertsFile(REF, hidden=64, verify=True)
    ps = json.loads((REF / "pieces.json").read_text())
    assert ef.layout == RecordLayout(ps["hidden"], ps["inter"], ps["gs"])
    assert ef.piece_offsets == ef.layout.offsets() and ef.record_bytes == ef.layout.record_bytes
    for L in range(ef.layers):
        for e in range(ef.experts):
            for j in range(len(PIECE_NAMES)):
                assert hashlib.sha256(ef.piece(L, e, j).tobytes()).hexdigest() == ps["sha256"][L][e][j]


def test_writer_reproduces_the_reference_file(tmp_path):
    ef = ExpertsFile(REF)
    s = write_experts_bin(tmp_path, ef.layers, ef.experts, ef.piece_sizes, lambda L: ef.layer_records(L))
    assert s["written_layers"] == [0, 1]
    assert (tmp_path / "experts.bin").read_bytes() == (REF / "experts.bin").read_bytes()
    mine = json.loads((tmp_path / "experts.manifest.json").read_text())
    theirs = json.loads((REF / "experts.manifest.json").read_text())
    assert {k: mine[k] for k in FORMAT_KEYS} == {k: theirs[k] for k in FORMAT_KEYS}
    assert mine["stamp"]["size"] == theirs["total_bytes"]
    assert not (tmp_path / "experts.bin.tmp").exists()
    assert write_experts_bin(tmp_path, ef.layers, ef.experts, ef.piece_sizes, None)["status"] == "already done"


def test_resume_after_a_crash_rewrites_only_the_missing_layer(tmp_path):
    ef = ExpertsFile(REF)
    write_experts_bin(tmp_path, ef.layers, ef.experts, ef.piece_sizes, lambda L: ef.layer_records(L))
    full = (tmp_path / "experts.bin").read_bytes()
    # crash after layer 0: the tmp file back in place, layer 1 missing from progress and damaged on disk
    (tmp_path / "experts.bin").rename(tmp_path / "experts.bin.tmp")
    (tmp_path / "experts.manifest.json").unlink()
    prog = json.loads((tmp_path / "experts.progress.json").read_text())
    prog.pop("1")
    (tmp_path / "experts.progress.json").write_text(json.dumps(prog))
    lb = ef.experts * ef.record_bytes
    with open(tmp_path / "experts.bin.tmp", "r+b") as f:
        f.seek(lb)
        f.write(b"\xff" * lb)
    s = write_experts_bin(tmp_path, ef.layers, ef.experts, ef.piece_sizes, lambda L: ef.layer_records(L))
    assert s["written_layers"] == [1]
    assert (tmp_path / "experts.bin").read_bytes() == full


def test_synthetic_records_round_trip(tmp_path):
    lay = RecordLayout(128, 64, 64)
    E = 32
    recs = {L: np.stack([synth.expert_record(lay, 3, L, e) for e in range(E)]) for L in range(3)}
    write_experts_bin(tmp_path, 3, E, [lay.w_bytes, lay.sb_bytes, lay.sb_bytes] * 3, lambda L: recs[L])
    ef = ExpertsFile(tmp_path, hidden=128, verify=True)
    assert ef.layout == lay
    for L in range(3):
        np.testing.assert_array_equal(ef.layer_records(L), recs[L])


def test_bad_files_are_refused(tmp_path):
    def copy(name):
        d = tmp_path / name
        shutil.copytree(REF, d)
        return d, json.loads((d / "experts.manifest.json").read_text())

    d, m = copy("layout")
    m["layout"] = "something-else"
    (d / "experts.manifest.json").write_text(json.dumps(m))
    with pytest.raises(ManifestError):
        ExpertsFile(d)
    d, m = copy("order")
    m["piece_names"] = m["piece_names"][::-1]
    (d / "experts.manifest.json").write_text(json.dumps(m))
    with pytest.raises(ManifestError):
        ExpertsFile(d)
    d, _ = copy("short")
    with open(d / "experts.bin", "r+b") as f:
        f.truncate(4096)
    with pytest.raises(ManifestError):
        ExpertsFile(d)
    d, _ = copy("corrupt")
    with open(d / "experts.bin", "r+b") as f:
        f.seek(16 * 6912 + 100)
        f.write(b"\x00\x01\x02")
    assert ExpertsFile(d).verify() == [1]
    with pytest.raises(ManifestError):
        ExpertsFile(d, verify=True)
    with pytest.raises(ManifestError):
        ExpertsFile(REF, hidden=96)            # piece sizes of a 64-wide model do not fit 96


def test_layout_from_piece_sizes_and_alignment_rule(tmp_path):
    for lay in (RecordLayout(2048, 512, 64), RecordLayout(2560, 640, 64), RecordLayout(2048, 512, 32)):
        assert layout_of([lay.w_bytes, lay.sb_bytes, lay.sb_bytes] * 3, lay.hidden) == lay
    assert RecordLayout(2560, 640, 64).record_bytes == 2_764_800
    lay = RecordLayout(64, 64, 64)
    with pytest.raises(ValueError, match="multiple of 4096"):
        write_experts_bin(tmp_path, 1, 3, [lay.w_bytes, lay.sb_bytes, lay.sb_bytes] * 3,
                          lambda L: np.zeros((3, lay.record_bytes), np.uint8))
