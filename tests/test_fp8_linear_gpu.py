"""Per-block FP8 training linear (forward, dgrad, wgrad) and the FSDP2 FP8
all-gather, against CPU references built from the same quantized operands."""

import os
import subprocess
import sys

import pytest
import torch

import oracle
from practice_cuda_b200.fp8_linear import FP8BlockLinear
from tests._util import assert_bmm_close, synthetic

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _ref_gemm(a, sa, qbm, b, sb, qbn):
    """fp32 per-128-K-group promotion reference for a 2-D GEMM."""
    return oracle.scaled_bmm_promoted_reference(a.unsqueeze(0), sa.unsqueeze(0), b.unsqueeze(0), sb.unsqueeze(0),
                                                qbm=qbm, qbk=128, qbn=qbn, out_dtype=torch.float32)[0]


@pytest.mark.parametrize("t,din,dout", [(256, 384, 512), (384, 256, 128)])
def test_fp8_linear_forward_backward(t, din, dout):
    x = synthetic((t, din), outliers=True, seed=1)
    w = synthetic((dout, din), std=0.02, seed=2, dtype=torch.float32)
    dy = synthetic((t, dout), std=0.1, seed=3)
    lin = FP8BlockLinear(din, dout, bias=False).cuda()
    with torch.no_grad():
        lin.weight.copy_(w)
    xg = x.cuda().requires_grad_(True)
    y = lin(xg)
    y.backward(dy.cuda())
    # CPU references from the oracle's quantization of the same tensors.
    qx, sx = oracle.per_block_quant(x, block_m=1, block_n=128)
    qw, sw = oracle.per_block_quant(w, block_m=128, block_n=128)
    y_ref = _ref_gemm(qx, sx, 1, qw.t(), sw.t(), 128)
    assert_bmm_close(y.float(), y_ref, "forward")
    qdy, sdy = oracle.per_block_quant(dy, block_m=1, block_n=128)
    dx_ref = _ref_gemm(qdy, sdy, 1, qw, sw, 128)
    assert_bmm_close(xg.grad.float(), dx_ref, "dgrad")
    qdyt, sdyt = oracle.per_block_quant(dy, block_m=128, block_n=1)
    qxt, sxt = oracle.per_block_quant(x, block_m=128, block_n=1)
    dw_ref = _ref_gemm(qdyt.t(), sdyt.t(), 1, qxt, sxt, 1)
    assert_bmm_close(lin.weight.grad.float(), dw_ref, "wgrad")
    # And close to the high-precision linear (fp8 quantization error only).
    y_hp = x.float() @ w.t()
    cos = torch.nn.functional.cosine_similarity(y.float().cpu().flatten(), y_hp.flatten(), dim=0)
    assert cos > 0.99


_FSDP_SCRIPT = r"""
import os, sys, torch
sys.path.insert(0, sys.argv[1])
import torch.distributed as dist
from torch.distributed.fsdp import fully_shard, MixedPrecisionPolicy
from practice_cuda_b200.llama import Llama, LlamaConfig
from practice_cuda_b200.fsdp_fp8 import enable_fp8_all_gather, FP8AllGatherWeight
from practice_cuda_b200.fp8_linear import BlockFP8Weight, FP8BlockLinear
os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=sys.argv[2], RANK="0", WORLD_SIZE="1")
torch.cuda.set_device(0)
dist.init_process_group("nccl", device_id=torch.device("cuda", 0))
cfg = LlamaConfig(n_layers=2, dim=256, n_heads=4, ffn_dim=512, vocab=1024, seq_len=128)
def build(fsdp):
    torch.manual_seed(0)
    m = Llama(cfg).cuda()
    m.init_weights(0)
    if fsdp:
        enable_fp8_all_gather(m)
        mp = MixedPrecisionPolicy(param_dtype=torch.bfloat16, reduce_dtype=torch.float32)
        for layer in m.layers:
            fully_shard(layer, mp_policy=mp)
        fully_shard(m, mp_policy=mp)
    return m
seen = []
orig = FP8BlockLinear.forward
def spy(self, x):
    seen.append(isinstance(self.weight, BlockFP8Weight))
    return orig(self, x)
FP8BlockLinear.forward = spy
tok = torch.randint(0, cfg.vocab, (1, cfg.seq_len), generator=torch.Generator().manual_seed(1)).cuda()
losses = {}
for fsdp in (True, False):
    m = build(fsdp)
    opt = torch.optim.AdamW(m.parameters(), lr=1e-3)
    ls = []
    for _ in range(3):
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=not fsdp):
            logits = m(tok[:, :-1])
        loss = torch.nn.functional.cross_entropy(logits.float().reshape(-1, cfg.vocab), tok[:, 1:].reshape(-1))
        loss.backward()
        opt.step(); opt.zero_grad()
        ls.append(loss.item())
    losses[fsdp] = ls
assert all(seen[: 2 * 7]), "FSDP unshard did not yield per-block FP8 weights"
print("losses", losses)
assert all(torch.isfinite(torch.tensor(v)).all() for v in losses.values())
assert losses[True][2] < losses[True][0]
assert abs(losses[True][0] - losses[False][0]) < 0.05 * abs(losses[False][0])
dist.destroy_process_group()
print("FSDP_FP8_OK")
"""


def test_fsdp2_fp8_all_gather_single_rank():
    """FSDP2 with the per-block FP8 all-gather on one rank (NCCL world 1):
    unsharded weights arrive as fp8 + scales, training steps run and the
    loss matches the same model without FSDP."""
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    r = subprocess.run([sys.executable, "-c", _FSDP_SCRIPT, ROOT, str(port)], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and "FSDP_FP8_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
