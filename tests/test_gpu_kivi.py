"""quant_dequant_kivi_k / _v (kivi_helpers.py:35-59) on the GPU against the
reference's outputs (tests/golden/kivi.npz): bit-exact in every dtype,
including the NaN of an all-zero fp16 channel / token."""

import json
import os

import numpy as np
import pytest
import torch

from conftest import load_pkg

pytestmark = pytest.mark.gpu
KIVI = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "kivi.npz"))
META = json.loads(str(KIVI["meta"]))
TD = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


@pytest.mark.parametrize("case", META, ids=[f"{c['dtype']}_b{c['bits']}_{c['key']}" for c in META])
def test_kivi_bit_exact(case):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    pkg = load_pkg()
    x = torch.from_numpy(KIVI[case["key"] + "_x"]).to(TD[case["dtype"]]).cuda()
    for fn, name in ((pkg.quant_dequant_kivi_k, "_k"), (pkg.quant_dequant_kivi_v, "_v")):
        got = fn(x, case["bits"]).float().cpu().numpy()
        np.testing.assert_array_equal(got, KIVI[case["key"] + name], err_msg=f"{case['key']}{name}")
