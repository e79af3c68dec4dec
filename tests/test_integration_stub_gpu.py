"""The ctypes binding printed in INTEGRATION.md (the stub a maintainer would add to the
reference's experiments/triton_paged_attention.py) runs as printed and returns what the
package's paged_gather_decode_attention returns."""

import re
from pathlib import Path

import pytest
import torch

import attention_b200 as spa

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _stub_namespace() -> dict:
    text = (ROOT / "INTEGRATION.md").read_text()
    section = text[text.index("### The ctypes binding"):]
    code = re.search(r"```python\n(.*?)```", section, re.S).group(1)
    code = code.replace('"attention_b200/libspa_b200.so"', repr(str(ROOT / "attention_b200" / "libspa_b200.so")))
    ns: dict = {}
    exec(compile(code, "INTEGRATION.md", "exec"), ns)
    return ns


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_integration_stub_matches_package(dtype):
    stub = _stub_namespace()["paged_gather_decode_attention"]
    g = torch.Generator(device="cuda").manual_seed(21)
    b, h, length, d, block, window = 2, 4, 64 * 12 + 128, 64, 64, 128
    q = (torch.randn(b, h, d, device="cuda", generator=g) * 0.5).to(dtype)
    k = (torch.randn(b, h, length, d, device="cuda", generator=g) * 0.5).to(dtype)
    v = (torch.randn(b, h, length, d, device="cuda", generator=g) * 0.5).to(dtype)
    sel = torch.tensor([[0, 5, 11], [3, 7, -1]], device="cuda")
    got = stub(q, k, v, sel, local_window=window, block_size=block)
    ref = spa.paged_gather_decode_attention(q, k, v, sel, local_window=window, block_size=block)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    assert spa.device_error_flags() == 0
