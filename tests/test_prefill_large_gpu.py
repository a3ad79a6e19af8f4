"""Row-sample parity at the sizes the benchmark measures.

Every configuration that bench.py or the design notes report a throughput for
is checked here against the CPU oracle: config 2 (32/8 heads, W=2048, S=128)
at N=131072 for every stride gamma, config 5 (64/8 heads, W=4096, S=128,
gamma=64) at N=131072 and N=1,048,576 (query offsets beyond 2^32 elements),
and the per-GPU shares of strong scaling (one and two KV groups), where the
dense rows run split over keys.  An output row depends only on its own query
row, its KV group and its anchor, so the oracle is fed one group at a time and
only the query rows it asks for are copied from the GPU.
"""

import pytest
import torch

from delta_attention_b200.rope import apply_rope, cos_sin
from oracle import delta_oracle as orc
from tests._helpers import assert_close

pytestmark = pytest.mark.gpu


def _inputs(s, H, Hkv, d, seed):
    """Seeded bf16 q/k/v on the GPU, drawn and rotated a few heads at a time
    (fp32 intermediates of a whole 1M-token tensor would not fit)."""
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(seed)
    cos, sin = cos_sin(torch.arange(s, device=dev), d, 500000.0)

    def draw(n_heads, rope):
        t = torch.empty(1, n_heads, s, d, dtype=torch.bfloat16, device=dev)
        for h0 in range(0, n_heads, 4):
            h1 = min(n_heads, h0 + 4)
            x = torch.randn(1, h1 - h0, s, d, generator=gen, device=dev) * 0.5
            t[:, h0:h1] = (apply_rope(x, cos, sin) if rope else x).bfloat16()
            del x
        return t

    return draw(H, True), draw(Hkv, True), draw(Hkv, False)


class _GroupRows:
    """q of one KV group as the oracle sees it ([1, G, s, d]); rows are copied
    from the GPU only when the oracle indexes them."""

    def __init__(self, q, h0, h1):
        self.q, self.h0, self.h1 = q, h0, h1
        self.shape = (q.shape[0], h1 - h0, q.shape[2], q.shape[3])

    def __getitem__(self, idx):
        b, h, r = idx
        assert b == slice(None) and h == slice(None)
        r = torch.as_tensor(r, dtype=torch.long)
        return self.q[:, self.h0:self.h1][:, :, r.to(self.q.device)].cpu()


def _sample_rows(s, gamma, window, sink, seed=0):
    cut_n = s % gamma + max(128, gamma)
    s_p = s - cut_n
    fixed = [0, 1, gamma - 1, gamma, gamma + 1, sink - 1, sink, window + sink + 3,
             s_p - gamma, s_p - gamma + 7, s_p - 1, s_p, s_p + 5, s - 1]
    g = torch.Generator().manual_seed(seed)
    rnd = torch.randint(0, s, (6,), generator=g).tolist()
    return torch.tensor(sorted({r for r in fixed + rnd if 0 <= r < s}))


CASES = [
    # name, s, H, Hkv, window, sink, gamma
    ("config2-g16", 131072, 32, 8, 2048, 128, 16),
    ("config2-g32", 131072, 32, 8, 2048, 128, 32),
    ("config2-g64", 131072, 32, 8, 2048, 128, 64),
    ("config2-g128", 131072, 32, 8, 2048, 128, 128),
    ("config5-128k", 131072, 64, 8, 4096, 128, 64),
    ("strong-1-group", 131072, 4, 1, 2048, 128, 64),
    ("strong-2-groups", 131072, 8, 2, 2048, 128, 64),
    ("config5-1m", 1048576, 64, 8, 4096, 128, 64),
]


@pytest.mark.parametrize("name,s,H,Hkv,window,sink,gamma", CASES, ids=[c[0] for c in CASES])
def test_large_prefill_row_sample(name, s, H, Hkv, window, sink, gamma):
    from delta_attention_b200 import ops
    d = 128
    G = H // Hkv
    q, k, v = _inputs(s, H, Hkv, d, seed=len(name) + gamma)
    out = ops.prefill(q, k, v, gamma=gamma, window=window, sink=sink, check=True)
    rows = _sample_rows(s, gamma, window, sink)
    got = out[:, rows.cuda()].cpu()
    del out
    for g in sorted({0, Hkv - 1}):
        qg = _GroupRows(q, g * G, (g + 1) * G)
        kg, vg = k[:, g:g + 1].cpu(), v[:, g:g + 1].cpu()
        ref = orc.delta_forward_rows(qg, kg, vg, rows, gamma, window, sink, dtype=torch.float32)
        assert_close(got[:, :, g * G:(g + 1) * G], ref, f"{name} group {g}")
