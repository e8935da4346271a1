"""The bounds-checked debug build (`_C_debug`, LK_DEBUG_BOUNDS=1).

It runs in a child process, since a process loads one of the two modules.  The
child builds a small paged fp8 KV cache and checks two things:
  * with valid block tables and slots, the debug build's decode attention and
    KV gather match the fp32 reference;
  * a block-table entry or a slot outside the cache is reported in the status
    word (code 5, index out of range), and its tokens are skipped, with no
    out-of-range access.
The regular build is never given a bad index.
"""
import json
import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu

CHILD = textwrap.dedent(r'''
    import json, math, sys
    import torch
    from lora_kernel_b200 import _ext
    from lora_kernel_b200.ops import serving as SV
    assert _ext.C().__name__.endswith("_C_debug"), _ext.C().__name__
    torch.manual_seed(0)
    dev = "cuda"
    Hq, Hkv, Dh, bs = 8, 2, 128, 16
    nblk, nseq, ctx = 64, 3, 100
    slots = nblk * bs
    kc = (torch.randn(slots, Hkv, Dh, device=dev) * 0.5).to(torch.float8_e4m3fn)
    vc = (torch.randn(slots, Hkv, Dh, device=dev) * 0.5).to(torch.float8_e4m3fn)
    ks = torch.rand(slots, Hkv, device=dev) + 0.5
    vs = torch.rand(slots, Hkv, device=dev) + 0.5
    need = (ctx + bs - 1) // bs
    bt = torch.stack([torch.randperm(nblk, device=dev)[:need] for _ in range(nseq)]).int().contiguous()
    lens = torch.full((nseq,), ctx, dtype=torch.int32, device=dev)
    q = torch.randn(nseq, Hq * Dh, device=dev).bfloat16()
    st = _ext.status(torch.device(dev))
    st.zero_()
    out = SV.decode_attention(q, kc, vc, ks, vs, bt, lens, bs, Hq, Hkv, Dh, kv_dtype="fp8", split_len=64)
    torch.cuda.synchronize()
    res = {"status_valid": int(st.item())}
    # fp32 reference
    K = kc.float() * ks[..., None]
    V = vc.float() * vs[..., None]
    errs = []
    for s in range(nseq):
        sl = (bt[s].long()[:, None] * bs + torch.arange(bs, device=dev)).reshape(-1)[:ctx]
        for h in range(Hq):
            g = h // (Hq // Hkv)
            sc = (K[sl, g] @ q[s, h * Dh:(h + 1) * Dh].float()) / math.sqrt(Dh)
            o = torch.softmax(sc, 0) @ V[sl, g]
            errs.append(((out[s, h * Dh:(h + 1) * Dh].float() - o).norm() / o.norm()).item())
    res["decode_err"] = max(errs)
    # kv_gather of valid slots
    sl = (bt[0].long()[:, None] * bs + torch.arange(bs, device=dev)).reshape(-1)[:ctx].int().contiguous()
    gath = SV.kv_gather(kc, vc, ks, vs, sl, Hkv, Dh, kv_dtype="fp8")
    torch.cuda.synchronize()
    refk = K[sl.long()].reshape(ctx, Hkv * Dh)
    res["gather_err"] = ((gath[:, :Hkv * Dh].float() - refk).norm() / refk.norm()).item()
    res["status_after_valid"] = int(st.item())
    # a block id past the cache: reported, its tokens skipped
    bad = bt.clone()
    bad[1, 2] = nblk + 7
    out_bad = SV.decode_attention(q, kc, vc, ks, vs, bad, lens, bs, Hq, Hkv, Dh, kv_dtype="fp8", split_len=64)
    torch.cuda.synchronize()
    res["status_bad_block"] = int(st.item())
    res["bad_block_output_finite"] = bool(torch.isfinite(out_bad.float()).all().item())
    res["other_seqs_unchanged"] = bool(torch.equal(out_bad[0], out[0]) and torch.equal(out_bad[2], out[2]))
    # a negative slot in a gather: reported, the row is zero
    st.zero_()
    sl_bad = sl.clone()
    sl_bad[5] = -3
    g2 = SV.kv_gather(kc, vc, ks, vs, sl_bad, Hkv, Dh, kv_dtype="fp8")
    torch.cuda.synchronize()
    res["status_bad_slot"] = int(st.item())
    res["bad_row_zero"] = bool((g2[5] == 0).all().item())
    res["good_rows_same"] = bool(torch.equal(g2[:5], gath[:5]) and torch.equal(g2[6:], gath[6:]))
    st.zero_()
    print("RESULT " + json.dumps(res))
''')


def test_debug_build_reports_bad_indices_without_touching_memory():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, LK_DEBUG_BOUNDS="1", PYTHONPATH=root)
    r = subprocess.run([sys.executable, "-c", CHILD], env=env, capture_output=True, text=True, timeout=600,
                       cwd=root)
    line = [x for x in r.stdout.splitlines() if x.startswith("RESULT ")]
    assert r.returncode == 0 and line, r.stdout[-2000:] + r.stderr[-4000:]
    res = json.loads(line[0][7:])
    assert res["status_valid"] == 0 and res["status_after_valid"] == 0, res
    assert res["decode_err"] < 3e-2, res
    assert res["gather_err"] < 1e-2, res
    assert res["status_bad_block"] == 5, res
    assert res["bad_block_output_finite"] and res["other_seqs_unchanged"], res
    assert res["status_bad_slot"] == 5 and res["bad_row_zero"] and res["good_rows_same"], res
