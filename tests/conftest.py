import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the native library")


@pytest.fixture(scope="session")
def attention_golden():
    z = np.load(os.path.join(GOLDEN, "attention.npz"))
    cases = {}
    for name in z["names"]:
        name = str(name)
        pre = name + "/"
        c = {k[len(pre):]: z[k] for k in z.files if k.startswith(pre)}
        Hq, Hkv, D, P, dense, is_fp16 = (int(x) for x in c["meta"])
        c.update(Hq=Hq, Hkv=Hkv, D=D, P=P, dense=bool(dense),
                 dtype="float16" if is_fp16 else "bfloat16",
                 scale_f=float(c["scale"][0]), softcap_f=float(c["softcap"][0]))
        cases[name] = c
    return cases


@pytest.fixture(scope="session")
def placement_golden():
    with open(os.path.join(GOLDEN, "placement.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def norm_rope_golden():
    return np.load(os.path.join(GOLDEN, "norm_rope.npz"))


@pytest.fixture(scope="session")
def prefill_golden():
    z = np.load(os.path.join(GOLDEN, "prefill.npz"))
    cases = {}
    for name in z["names"]:
        name = str(name)
        pre = name + "/"
        c = {k[len(pre):]: z[k] for k in z.files if k.startswith(pre)}
        Hq, Hkv, D, P, S, is_fp16 = (int(x) for x in c["meta"])
        c.update(Hq=Hq, Hkv=Hkv, D=D, P=P, S=S, dtype="float16" if is_fp16 else "bfloat16",
                 softcap_f=float(c["softcap"][0]))
        cases[name] = c
    return cases
