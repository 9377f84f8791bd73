"""The bounds-checked debug build (``GLM53_BOUNDS=1``: ``glm53_C_bounds``), run in a child process.

Negative cases: each guarded kernel gets one index that is out of range for the tensor it indexes (a token id, an
MLA cache slot read through the selection, a KDA state and conv slot, a DSA page, an MoE token row and expert id).
The kernel must skip the access, record (code, index, limit) and leave the context usable; every input is small
and every other index in range, so nothing outside the guarded accesses reads past a buffer.

Positive case: the tiny proxy prefilled in chunks of 1, 17, 64 and 130 rows (tile edges of the decode and prefill
kernels), then verify windows of 1 and 8 rows; no index may be out of range, every guard band around the
runtime's scratch must be intact, and the logits must agree across the chunkings.
"""

import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_CHILD = r'''
import json, os, sys
sys.path.insert(0, os.environ["G53_ROOT"])
import torch
from glm53.ops import _ext
assert _ext.BOUNDS and _ext.NAME == "glm53_C_bounds", (_ext.BOUNDS, _ext.NAME)
C = _ext.require()
DEV = "cuda"
out = {}

def status(tag):
    torch.cuda.synchronize()
    en, fails = C.bounds_status()
    C.bounds_reset()
    out[tag] = dict(enabled=en, fails=[list(f) for f in fails])

status("clean")
g = torch.Generator(device=DEV).manual_seed(0)

# 1. embedding: ids V and -1 of a V-row table
V, D, S = 64, 256, 4
table = torch.randn(V, D, device=DEV, generator=g).to(torch.bfloat16)
X = torch.full((4, S, D), 7.0, device=DEV, dtype=torch.bfloat16)
ids = torch.tensor([3, V, -1, 5], dtype=torch.int32, device=DEV)
C.embed(ids, table, X)
status("embed")
out["embed_ok"] = bool(torch.equal(X[0, 0], table[3]) and torch.equal(X[3, 0], table[5])
                       and bool((X[1:3] == 7.0).all()))

# 2. sparse MLA: two selected slots out of range (the limit itself and far past it), both kernels
L, H, R, NS, MS = 512, 16, 2, 256, 128
q_lat = (torch.randn(R, H, L, device=DEV, generator=g) * 0.5).to(torch.bfloat16)
kv = (torch.randn(NS, L, device=DEV, generator=g) * 40).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
scale = torch.rand(NS, device=DEV, generator=g) * 0.02 + 0.001
sel = torch.stack([torch.randperm(NS, device=DEV, generator=g)[:MS] for _ in range(R)]).to(torch.int32)
sel[1, 5] = NS
sel[1, 77] = 100000
cnt = torch.full((R,), MS, dtype=torch.int32, device=DEV)
for tc in (0, 1):
    part_o = torch.empty(R * H * L, device=DEV)
    part_ml = torch.empty(R * H * 2, device=DEV)
    o = torch.full_like(q_lat, float("nan"))
    C.mla_decode(q_lat, None, 0, 0, kv, scale, None, sel, cnt, 0, 0.05, 1, part_o, part_ml, o, tc)
    status(f"mla_tc{tc}")
    out[f"mla_tc{tc}_finite"] = bool(torch.isfinite(o.float()).all())

# 3. KDA: recurrent form with an out-of-range input state, conv with an out-of-range conv slot
T, KH, Dh = 8, 2, 64
HD = KH * Dh
ldp = (3 * HD + 2 * Dh + KH + 63) // 64 * 64
proj = (torch.randn(T, ldp, device=DEV, generator=g) * 0.5).to(torch.bfloat16)
qkv = torch.randn(T, 3 * HD, device=DEV, generator=g).to(torch.bfloat16)
f = torch.randn(T, HD, device=DEV, generator=g).to(torch.bfloat16)
a_log = torch.log(torch.rand(KH, device=DEV, generator=g) * 15 + 1)
dt_bias = torch.randn(HD, device=DEV, generator=g) * 0.5
Sp = torch.zeros(2, KH, Dh, Dh, device=DEV)
seq = torch.tensor([[0], [T], [2], [1], [0]], dtype=torch.int32, device=DEV)
o_raw = torch.full((T, HD), 3.0, device=DEV)
C.kda_recurrent(proj, seq, f, qkv, a_log, dt_bias, Sp, o_raw, KH, Dh, 3 * HD + 2 * Dh, -5.0)
status("kda_state")
out["kda_state_untouched"] = bool((Sp == 0).all() and (o_raw == 3.0).all())
conv_w = torch.randn(3 * HD, 4, device=DEV, generator=g)
conv_pool = torch.zeros(2, 3, 3 * HD, device=DEV, dtype=torch.bfloat16)
seqc = torch.tensor([[0], [T], [0], [0], [5]], dtype=torch.int32, device=DEV)
qkv2 = torch.full((T, 3 * HD), 9.0, device=DEV, dtype=torch.bfloat16)
C.kda_conv(proj, seqc, T, conv_w, conv_pool, qkv2, KH, Dh)
status("kda_conv")
out["kda_conv_untouched"] = bool((qkv2 == 9.0).all())

# 4. DSA indexer logits: one page of the page table far past the pool cache, both kernels
ID, IH, kpool, bs, pages, nb = 128, 4, 4, 64, 40, 24
pos = list(range(1500, 1508))
bt = torch.randperm(pages, generator=torch.Generator().manual_seed(1))[:nb].to(torch.int32).view(1, nb).to(DEV)
bt[0, 3] = 100000
raw = torch.randint(0, 256, (pages * bs // kpool, ID), generator=g, device=DEV, dtype=torch.int32)
raw[(raw == 0x7F) | (raw == 0xFF)] = 0
pool_cache = raw.to(torch.uint8)
pool_scale = torch.ones(pages * bs // kpool, device=DEV)
iproj = torch.randn(len(pos), ID + IH + ID, device=DEV, generator=g)
qi = torch.randn(len(pos), IH * ID, device=DEV, generator=g).to(torch.bfloat16)
positions = torch.tensor(pos, dtype=torch.int32, device=DEV)
row_seq = torch.zeros(len(pos), dtype=torch.int32, device=DEV)
for tc in (False, True):
    lg = torch.zeros(len(pos), nb * bs // kpool, device=DEV)
    C.dsa_logits(iproj, qi, torch.ones(ID, device=DEV), pool_cache, pool_scale, positions, bt, row_seq, bs, IH,
                 kpool, lg, tc)
    status(f"dsa_tc{int(tc)}")
    out[f"dsa_tc{int(tc)}_finite"] = bool(torch.isfinite(lg).all())

# 5. MoE rotated inputs: a pair whose token row is past x, a pair whose expert is past the experts
K, E, Tm = 256, 4, 3
x = torch.randn(Tm, K, device=DEV, generator=g).to(torch.bfloat16)
suh = torch.ones(E, K, device=DEV, dtype=torch.float16)
pt = torch.tensor([0, Tm, 1, 2], dtype=torch.int32, device=DEV)
pe = torch.tensor([0, 1, E + 3, 2], dtype=torch.int32, device=DEV)
xg = torch.full((4, K), 5.0, device=DEV, dtype=torch.float16)
xu = torch.full((4, K), 5.0, device=DEV, dtype=torch.float16)
C.exl3_rot_in(x, suh, suh, pt, pe, xg, xu)
status("moe_rot_in")
out["moe_skipped_rows_untouched"] = bool((xg[1:3] == 5.0).all() and not (xg[0] == 5.0).all())

# 6. the tiny proxy at tile-edge chunk sizes: nothing out of range, guard bands intact, logits agree
sys.path.insert(0, os.environ["G53_ROOT"])
import glm53
from glm53.models import weights as W
from glm53.models.runtime import Runtime, RuntimeConfig
from glm53.models.session import Sequence
from glm53.utils import canary
from tests.test_gpu_kernels import _to_dev
cfg = glm53.tiny_config()
w = _to_dev(W.prepare(W.DictSource(W.random_checkpoint(cfg, seed=0)), cfg))
prompt = torch.randint(0, cfg.vocab, (150,), generator=torch.Generator().manual_seed(0)).tolist()
ref = None
cos = {}
for chunk in (64, 1, 17, 130):
    rt = Runtime(w, RuntimeConfig(max_rows=130, kv_slots=1024, block_size=64, max_blocks=16))
    sq = Sequence(rt)
    lg = [sq.prefill(prompt, chunk=chunk)[0].float()]
    lg.append(sq.verify([3])[0].float())
    sq.commit(1)
    lg.append(sq.verify([5, 6, 7, 8, 9, 10, 11, 12])[-1].float())
    sq.commit(8)
    v = torch.cat(lg)
    if ref is None:
        ref = v
    cos[chunk] = torch.nn.functional.cosine_similarity(v, ref, dim=0).item()
    status(f"model_chunk{chunk}")
    out[f"guards_chunk{chunk}"] = dict(buffers=len(rt.scratch), bad=canary.check_all())
out["model_cos"] = cos
print("RESULT " + json.dumps(out))
'''


@pytest.fixture(scope="module")
def bounds_run():
    env = dict(os.environ, GLM53_BOUNDS="1", G53_ROOT=ROOT)
    env.pop("PYTEST_CURRENT_TEST", None)
    p = subprocess.run([sys.executable, "-c", _CHILD], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=1500)
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("RESULT ")]
    assert p.returncode == 0 and lines, (p.returncode, p.stdout[-3000:], p.stderr[-3000:])
    return json.loads(lines[-1][len("RESULT "):])


def _one(r, tag, code, indices):
    st = r[tag]
    assert st["enabled"], tag
    assert len(st["fails"]) >= 1, (tag, st)
    codes = {f[0] for f in st["fails"]}
    assert codes == {code}, (tag, st)
    assert any(f[1] in indices for f in st["fails"]), (tag, st)


def test_clean_start(bounds_run):
    assert bounds_run["clean"] == {"enabled": True, "fails": []}


def test_embed_out_of_range(bounds_run):
    _one(bounds_run, "embed", 1, {64, -1})
    assert sum(f[3] for f in bounds_run["embed"]["fails"]) >= 2       # both bad rows (every column block) counted
    assert bounds_run["embed_ok"]


@pytest.mark.parametrize("tc", [0, 1])
def test_mla_selection_out_of_range(bounds_run, tc):
    _one(bounds_run, f"mla_tc{tc}", 3, {256, 100000})
    assert bounds_run[f"mla_tc{tc}_finite"]


def test_kda_slots_out_of_range(bounds_run):
    _one(bounds_run, "kda_state", 5, {2})
    assert bounds_run["kda_state_untouched"]
    _one(bounds_run, "kda_conv", 5, {5})
    assert bounds_run["kda_conv_untouched"]


@pytest.mark.parametrize("tc", [0, 1])
def test_dsa_page_out_of_range(bounds_run, tc):
    st = bounds_run[f"dsa_tc{tc}"]
    assert {f[0] for f in st["fails"]} == {4}, st
    assert bounds_run[f"dsa_tc{tc}_finite"]


def test_moe_rows_and_experts_out_of_range(bounds_run):
    st = bounds_run["moe_rot_in"]
    assert {f[0] for f in st["fails"]} <= {6, 7} and st["fails"], st
    assert bounds_run["moe_skipped_rows_untouched"]


@pytest.mark.parametrize("chunk", [1, 17, 64, 130])
def test_model_tile_edges_clean(bounds_run, chunk):
    assert bounds_run[f"model_chunk{chunk}"]["fails"] == [], bounds_run[f"model_chunk{chunk}"]
    g = bounds_run[f"guards_chunk{chunk}"]
    assert g["buffers"] > 50 and g["bad"] == [], g
    assert bounds_run["model_cos"][str(chunk)] > 0.99, bounds_run["model_cos"]
