"""CPU: the .ssm container side of the boundary (no GPU calls).

The C++ planner in liblssm_cuda.so must reproduce, byte for byte, the header +
tensor index the reference's tools/ssm_format.py:plan_layout writes for the
mamba2-130m state_dict (fixtures made by tests/golden/make_golden.py), i.e. the
known answers of tests/test_mmap_loader.cpp:64-95 (219 tensors, embedding payload
at 17600, in_proj (3352, 768), 64-byte aligned payloads). The C++ parser must
accept the reference-written tiny .ssm files and reject corrupt ones with the
reference loader's messages (src/core/ssm_loader.cpp:56-137).
"""

import ctypes as C
import json
import struct

import numpy as np
import pytest

import lssm
import pyoracle as po


def hp130m():
    return lssm.hparams(d_model=768, n_layer=24, d_state=128, d_conv=4, expand=2, vocab_size=50288, n_heads=24,
                        d_head=64, chunk_size=256, n_groups=1)


@pytest.mark.parametrize("quant", ["fp16", "int4"])
def test_plan_matches_reference_layout(golden, quant):
    ref = (golden / f"layout_130m_{quant}.bin").read_bytes()
    table = json.loads((golden / f"layout_130m_{quant}.json").read_text())
    hp = hp130m()
    buf = C.create_string_buffer(len(ref) + 64)
    doff, total = C.c_uint64(), C.c_uint64()
    n = lssm.lib().lssm_plan_layout(C.byref(hp), 1 if quant == "int4" else 0, C.cast(buf, C.c_void_p), len(buf),
                                    C.byref(doff), C.byref(total))
    assert n == len(ref)
    assert buf.raw[:n] == ref
    assert doff.value == table["data_offset"] == 17600
    hdr, tensors = po.parse_ssm(ref + b"\0" * (total.value - len(ref)))
    assert hdr.n_tensors == table["n_tensors"] == 219
    emb = tensors["backbone.embeddings.weight"]
    assert emb.offset == 17600 and emb.shape == (50288, 768) and emb.nbytes == 50288 * 768 * 2
    ip = tensors["backbone.layers.12.mixer.in_proj.weight"]
    assert ip.shape == (3352, 768) and ip.offset % 64 == 0
    for t in table["tensors"]:
        assert tensors[t["name"]].offset == t["offset"] and tensors[t["name"]].nbytes == t["nbytes"]


@pytest.mark.parametrize("name", ["tinyA_fp16", "tinyA_int4", "tinyB_fp16", "tinyB_int4"])
def test_parse_reference_written_files(golden, name):
    data = (golden / f"{name}.ssm").read_bytes()
    hp = lssm.HParams()
    nt = C.c_uint32()
    err = C.create_string_buffer(512)
    rc = lssm.lib().lssm_parse_header(data, len(data), C.byref(hp), C.byref(nt), err, 512)
    assert rc == 0, err.value
    ph, tensors = po.parse_ssm(data)
    assert nt.value == ph.n_tensors == len(tensors)
    assert (hp.d_model, hp.n_layer, hp.n_groups, hp.vocab_size) == (ph.d_model, ph.n_layer, ph.n_groups, ph.vocab_size)


def _parse_err(data: bytes) -> str:
    err = C.create_string_buffer(512)
    rc = lssm.lib().lssm_parse_header(data, len(data), None, None, err, 512)
    assert rc != 0
    return err.value.decode()


def test_parse_rejects_corrupt_files(golden):
    data = bytearray((golden / "tinyB_fp16.ssm").read_bytes())
    assert "too small" in _parse_err(bytes(data[:50]))
    bad = bytearray(data); bad[0:4] = b"XSSM"
    assert "bad magic" in _parse_err(bytes(bad))
    bad = bytearray(data); bad[4:8] = struct.pack("<I", 2)
    assert "unsupported version" in _parse_err(bytes(bad))
    bad = bytearray(data); bad[8:12] = struct.pack("<I", 95)
    assert "header_size" in _parse_err(bytes(bad))
    # corrupt the first tensor's nbytes
    bad = bytearray(data); off = 96 + 24
    bad[off:off + 8] = struct.pack("<Q", struct.unpack("<Q", bad[off:off + 8])[0] + 2)
    assert "nbytes" in _parse_err(bytes(bad)) or "overflows" in _parse_err(bytes(bad))
    # rank 0
    bad = bytearray(data); bad[96 + 4:96 + 8] = struct.pack("<I", 0)
    assert "rank" in _parse_err(bytes(bad))
    # truncated payload
    assert "overflows" in _parse_err(bytes(data[: len(data) - 4096]))
