"""The C ABI library on any machine: it loads, exports every declared entry point, and fails loudly without a GPU."""
import ctypes
import glob
import os
import re

import pytest

from conftest import ROOT


def declared():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        names += re.findall(r"^\s*(?:int|const char\s*\*)\s+(laya_\w+)\s*\(", open(h).read(), re.M)
    return names


def test_header_declares_the_boundary():
    names = declared()
    for n in ["laya_ctx_create", "laya_upload_tensor", "laya_upload_q8_0", "laya_q8_0_linear", "laya_decision_forward",
              "laya_last_error", "laya_trainer_create", "laya_train_forward", "laya_train_backward",
              "laya_train_objective", "laya_train_clip_and_step", "laya_train_comm_init", "laya_decoder_create",
              "laya_decoder_upload", "laya_decoder_upload_q8_0", "laya_decoder_forward", "laya_decoder_logits"]:
        assert n in names


def test_library_exports_every_declared_symbol():
    import laya_b200
    L = laya_b200.lib()
    missing = [n for n in declared() if not hasattr(L, n)]
    assert not missing, missing
    assert L.laya_version().startswith(b"laya_b200")


def test_no_cpu_fallback_without_a_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("this machine has a GPU")
    import laya_b200
    with pytest.raises(laya_b200.LayaError):
        laya_b200.Context(laya_b200.base_desc(max_tokens=128, max_items=4, max_markers=16))


@pytest.mark.parametrize("header,struct,cls", [("laya_b200.h", "laya_model_desc", "ModelDesc"),
                                                ("laya_train.h", "laya_train_desc", "TrainDesc"),
                                                ("laya_train.h", "laya_rlcd_desc", "RlcdDesc"),
                                                ("laya_decoder.h", "laya_decoder_desc", "DecoderDesc")])
def test_struct_layouts_match_the_headers(tmp_path, header, struct, cls):
    """The ctypes mirrors of the C ABI structs have the C compiler's size and field offsets."""
    import subprocess
    import laya_b200
    C = getattr(laya_b200, cls)
    fields = [f for f, _ in C._fields_]
    src = tmp_path / "desc.c"
    src.write_text(f'#include <stdio.h>\n#include <stddef.h>\n#include "{header}"\nint main(void){{printf("%zu", sizeof({struct}));'
                   + "".join(f'printf(" %zu", offsetof({struct}, {f}));' for f in fields) + "return 0;}\n")
    exe = tmp_path / "desc"
    subprocess.check_call(["gcc", "-I" + os.path.join(ROOT, "include"), str(src), "-o", str(exe)])
    out = [int(v) for v in subprocess.check_output([str(exe)]).split()]
    assert out[0] == ctypes.sizeof(C)
    assert out[1:] == [getattr(C, f).offset for f in fields]


def test_trainer_fails_loudly_without_a_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("this machine has a GPU")
    import laya_b200
    with pytest.raises(laya_b200.LayaError):
        laya_b200.Trainer(laya_b200.base_desc(max_tokens=128, max_items=4, max_markers=16))


def test_invalid_geometry_is_an_argument_error():
    import laya_b200
    with pytest.raises(laya_b200.LayaArgumentError):
        laya_b200.Context(laya_b200.base_desc(heads=7))


def test_decoder_fails_loudly_without_a_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("this machine has a GPU")
    import laya_b200
    with pytest.raises(laya_b200.LayaError):
        laya_b200.Qwen35Model(laya_b200.decoder_desc(["linear", "full"], max_tokens=64, max_seqs=2))


def test_decoder_invalid_geometry_is_an_argument_error():
    import laya_b200
    with pytest.raises(laya_b200.LayaArgumentError):
        laya_b200.Qwen35Model(laya_b200.decoder_desc(["linear"], lin_v_heads=3, lin_k_heads=2))
    with pytest.raises(laya_b200.LayaArgumentError):
        laya_b200.Qwen35Model(laya_b200.decoder_desc(["full"], head_dim=96))


def test_temperature_fit_through_the_abi_is_the_oracle():
    """laya_fit_temperatures (TemperatureFitting.Fit) is host code: on CPU it equals the oracle restatement bit for
    bit and recovers the reference's known temperature (TrainingTests.cs:84-105)."""
    import numpy as np
    import laya_b200
    from oracle.train import fit_temperatures, softmax_f32
    rng = np.random.default_rng(7)
    samples = []
    for i in range(420):
        k = [2, 4, 7, 12][i % 4]
        q = [0, 1, 2][i % 3] if i < 400 else 0
        z = (rng.random(k) * 8 - 4).astype(np.float32)
        samples.append((q, z, softmax_f32(z / np.float32(2))))
    got = laya_b200.fit_temperatures(samples, 30)
    want = fit_temperatures(samples, 30)
    assert [np.float32(v) for v in got[0]] == [np.float32(v) for v in want[0]]
    assert {k: np.float32(v) for k, v in got[1].items()} == {k: np.float32(v) for k, v in want[1].items()}
    assert got[2] == want[2]
    one = [s for s in samples if s[0] == 0 and len(s[1]) == 4][:200]
    t, b, c = laya_b200.fit_temperatures(one, 30)
    assert abs(t[0] - 2.0) < 1e-3 and abs(t[2] - 1.2) < 1e-6 and abs(b["choice:3-5"] - 2.0) < 1e-3
