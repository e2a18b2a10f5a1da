"""The readers of the reference's exported model files (host only, no GPU):
synthetic model directories written in the exporter's layout decode back into
exactly the fp32 weight streams the layers load (fp16-stored weights as their
fp16 values)."""
from __future__ import annotations

import numpy as np
import pytest

import ncnn_files
import s2b200
from s2b200 import synth


@pytest.mark.parametrize("shared,last,shifted,storage", [(False, False, True, "fp16"), (True, True, False, "fp16"),
                                                          (False, False, False, "fp32")])
def test_block_files_round_trip(tmp_path, shared, last, shifted, storage):
    dim, heads, mlp = 256, 2, 384
    w = synth.block_weights(dim, heads, mlp, shared, seed=5)
    expect = ncnn_files.write_block(tmp_path, 7, w, dim, heads, mlp, shared, last, shifted, storage)
    p, got = s2b200.read_ncnn_block(tmp_path / "seedvr2_dit_block_07.ncnn.param",
                                    tmp_path / "seedvr2_dit_block_07.ncnn.bin")
    assert (p["block_index"], p["shared"], p["last"], p["shifted"], p["dim"], p["heads"], p["mlp_hidden"]) == \
        (7, int(shared), int(last), int(shifted), dim, heads, mlp)
    assert abs(p["eps"] - 1e-5) < 1e-12
    assert np.array_equal(got, expect)


def test_head_files_round_trip(tmp_path):
    dim, tc = 128, 320
    wi = synth.dit_input_weights(dim, 33, tc, 256)
    ei = ncnn_files.write_input(tmp_path, wi, dim, tc)
    p, got = s2b200.read_ncnn_input(tmp_path / "seedvr2_dit_input.ncnn.param", tmp_path / "seedvr2_dit_input.ncnn.bin")
    assert (p["dim"], p["video_channels"], p["text_channels"], p["sinusoidal_dim"], p["embedding_dim"]) == \
        (dim, 33, tc, 256, 6 * dim)
    assert np.array_equal(got, ei)
    wo = synth.dit_output_weights(dim)
    eo = ncnn_files.write_output(tmp_path, wo, dim)
    p, got = s2b200.read_ncnn_output(tmp_path / "seedvr2_dit_output.ncnn.param",
                                     tmp_path / "seedvr2_dit_output.ncnn.bin")
    assert (p["dim"], p["out_channels"]) == (dim, 16)
    assert np.array_equal(got, eo)


def test_bad_files_are_rejected(tmp_path):
    dim, heads, mlp = 128, 1, 128
    w = synth.block_weights(dim, heads, mlp, True, seed=1)
    ncnn_files.write_block(tmp_path, 0, w, dim, heads, mlp, True, False, False)
    par, binp = tmp_path / "seedvr2_dit_block_00.ncnn.param", tmp_path / "seedvr2_dit_block_00.ncnn.bin"
    data = binp.read_bytes()
    binp.write_bytes(data[:-8])                                  # truncated
    with pytest.raises(s2b200.S2Error) as e:
        s2b200.read_ncnn_block(par, binp)
    assert e.value.status == s2b200.S2_INVALID_ARGUMENT
    binp.write_bytes(data + b"\0\0\0\0")                         # trailing bytes
    with pytest.raises(s2b200.S2Error):
        s2b200.read_ncnn_block(par, binp)
    bad = bytearray(data)
    bad[6 * dim * 4:6 * dim * 4 + 4] = (0x000D4B38).to_bytes(4, "little")   # an int8 tag
    binp.write_bytes(bytes(bad))
    with pytest.raises(s2b200.S2Error) as e:
        s2b200.read_ncnn_block(par, binp)
    assert e.value.status == s2b200.S2_UNSUPPORTED
    par.write_text("123\n")
    with pytest.raises(s2b200.S2Error):
        s2b200.read_ncnn_block(par, binp)
