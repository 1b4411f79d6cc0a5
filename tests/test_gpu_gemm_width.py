"""The CTA-pair INT8 GEMM in its three tile widths (256 x 256, 256 x 192, 256 x 128).

The library picks the width per launch from the tile count (narrow tiles when
the wide ones would leave most of a wave of SM pairs idle); QI_GEMM_PAIR_BN
forces one.  Every width must give exact INT32 accumulators and the same
dequantized (+ GELU / gated residual) outputs bit for bit, so a child process
per width runs the same seeded problems and the parent compares digests."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(os.path.dirname(HERE), "qwen-image.cu_b200")

# rows >= 512 run on CTA pairs; ragged M and N, K from 128 to 12288
SHAPES = [(512, 256, 128), (700, 544, 8192), (1000, 3072, 12288), (1786, 3072, 3072), (513, 12288, 3072),
          (2049, 9216, 3072)]

CHILD = r"""
import hashlib, json, sys
sys.path.insert(0, sys.argv[1])
import torch
import qib200 as Q
torch.cuda.set_device(0)
shapes = json.loads(sys.argv[2])
res = {}
for M, N, K in shapes:
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    a = torch.randint(-128, 128, (M, K), dtype=torch.int8, device="cuda", generator=g)
    w = torch.randint(-128, 128, (N, K), dtype=torch.int8, device="cuda", generator=g)
    out = Q.linear_i8(a, torch.ones(M, device="cuda"), w, torch.ones(N, device="cuda"))
    exact = (a.double() @ w.double().T).float()
    ok = bool(torch.equal(out, exact))
    sa = torch.rand(M, device="cuda", generator=g) * 1e-3
    sw = torch.rand(N, device="cuda", generator=g) * 1e-3
    b = (torch.rand(N, device="cuda", generator=g) - 0.5).to(torch.bfloat16)
    gate = torch.rand(N, device="cuda", generator=g) - 0.5
    resid = torch.randn(M, N, device="cuda", generator=g)
    h = hashlib.sha256()
    for epi in (Q.EPI_STORE, Q.EPI_GELU, Q.EPI_RESIDUAL):
        o = resid.clone() if epi == Q.EPI_RESIDUAL else None
        y = Q.linear_i8(a, sa, w, sw, b, epi, gate=gate if epi == Q.EPI_RESIDUAL else None, out=o)
        torch.cuda.synchronize()
        h.update(y.cpu().numpy().tobytes())
    res[f"{M}x{N}x{K}"] = [ok, h.hexdigest()]
print(json.dumps(res))
"""


def _run(width):
    env = dict(os.environ, QI_GEMM_PAIR_BN=str(width))
    r = subprocess.run([sys.executable, "-c", CHILD, PKG, json.dumps(SHAPES)], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_pair_tile_widths_agree_bit_for_bit():
    runs = {w: _run(w) for w in (256, 192, 128)}
    for key in runs[256]:
        for w, r in runs.items():
            assert r[key][0], f"{key}: {w}-wide tiles, accumulators not exact"
            assert r[key][1] == runs[256][key][1], f"{key}: {w}-wide tile outputs differ from the 256-wide ones"
