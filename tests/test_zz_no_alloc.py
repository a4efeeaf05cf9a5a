"""vg_k_attention_noalloc (scratch in a fixed library buffer, no device allocation) against
vg_k_attention (temporary stream-ordered scratch) and against the oracle's attention on the same
inputs. The file sorts last so the entry point also runs after every other GPU test has used the
device; it passes alone too."""
import numpy as np
import pytest

from conftest import assert_close
from oracle import oracle as O
from voxgen_b200 import api

pytestmark = pytest.mark.gpu

VG_ERANGE = -5


def _check(rc):
    assert rc == 0, f"status {rc}"


@pytest.mark.parametrize("heads,kv_heads,head_dim,ctx,pos", [
    (16, 2, 128, 4096, 4095),   # the BaseLM backbone shape at the end of its context
    (16, 2, 128, 4096, 1023),
    (8, 8, 64, 700, 333),
    (4, 1, 256, 64, 0),
    (32, 1, 128, 8192, 8191),   # 128 chunks of one KV head: 16 clusters merged per head
])
def test_noalloc_matches_allocating_entry_point(heads, kv_heads, head_dim, ctx, pos):
    import torch
    rng = np.random.default_rng(heads * 131 + ctx + pos)
    k_hm = rng.standard_normal((kv_heads, ctx, head_dim)).astype(np.float16)  # device layout
    v_hm = rng.standard_normal((kv_heads, ctx, head_dim)).astype(np.float16)
    # the oracle takes the reference layout [ctx][kv_heads * head_dim]
    k_ref = np.ascontiguousarray(k_hm.transpose(1, 0, 2).reshape(ctx, kv_heads * head_dim))
    v_ref = np.ascontiguousarray(v_hm.transpose(1, 0, 2).reshape(ctx, kv_heads * head_dim))
    kd, vd = torch.from_numpy(k_hm).cuda(), torch.from_numpy(v_hm).cuda()
    L = api.lib()
    for call in range(2):  # two consecutive calls: the merge counters must be clean for the second
        qh = (rng.standard_normal(heads * head_dim) * 0.3).astype(np.float32)
        q = torch.from_numpy(qh).cuda()
        want = torch.full((heads * head_dim,), float("nan"), dtype=torch.float32, device="cuda")
        got = torch.full_like(want, float("nan"))
        _check(L.vg_k_attention(q.data_ptr(), kd.data_ptr(), vd.data_ptr(), heads, kv_heads, head_dim, ctx, pos,
                                want.data_ptr(), None))
        _check(L.vg_k_attention_noalloc(q.data_ptr(), kd.data_ptr(), vd.data_ptr(), heads, kv_heads, head_dim,
                                        ctx, pos, got.data_ptr(), None))
        torch.cuda.synchronize()
        got_h = got.cpu().numpy()
        assert_close(got_h, want.cpu().numpy(), what=f"noalloc attention call {call} vs vg_k_attention")
        oracle, _ = O.attention(qh, k_ref.view(np.uint16), v_ref.view(np.uint16), heads, kv_heads, head_dim, pos)
        assert_close(got_h, oracle, what=f"noalloc attention call {call} vs the oracle")


def test_noalloc_rejects_oversize_scratch():
    import torch
    q = torch.zeros(64 * 128, dtype=torch.float32, device="cuda")
    kv = torch.zeros(16, dtype=torch.float16, device="cuda")
    out = torch.zeros_like(q)
    # 64 heads of 128 over 64 K/V heads at 131072 positions need 64*256*130*4 bytes of partials
    rc = api.lib().vg_k_attention_noalloc(q.data_ptr(), kv.data_ptr(), kv.data_ptr(), 64, 64, 128, 131072, 5,
                                          out.data_ptr(), None)
    assert rc == VG_ERANGE
    torch.cuda.synchronize()
