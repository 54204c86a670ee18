"""The drop-in, run: torchretrieve's own modules with their op namespace repointed to
``retrieve_b200.ops`` (the one-line change of retrieve/src/retrieve/interfaces.py:25), against
the same modules on the reference's ``"torch"`` backend, on the same seeded inputs.

The reference package is imported from its install under ``baseline/_ref`` (the reference's
``pip install --target``); without it every test here is skipped. CPU tests check that each op
the modules call exists in ``retrieve_b200.ops`` with the reference's parameter names. GPU tests
run ``ExactAttributeFilter``, ``LiNRV1`` (with and without the filter), ``LiNRV2``, ``LiNRV3``,
``OneBitKNN`` and ``SimHashKNN``: integer results bit for bit (masks, compactions, Hamming
scores), float scores within 1e-2 relative and recall@k >= 0.999 (the north star's tolerance);
and ``SilverTorch(backend="cuda")`` served by ``torch.ops.st.*`` from this library, against the
CPU restatement of ``st::search`` on the module's own index buffers.
"""

from __future__ import annotations

import importlib
import inspect
import sys
import types
from pathlib import Path

import numpy as np
import pytest
import torch

REF_SITE = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
pytestmark = pytest.mark.skipif(not (REF_SITE / "retrieve").is_dir(),
                                reason="the reference package is not installed under baseline/_ref")

OPS = ("clause_compact", "clause_mask", "clause_mask_scores", "fused_masked_knn_topk", "gemv_scores",
       "oporp_1bit_match_topk_full", "oporp_1bit_match_topk_indirect")


def _retrieve():
    if str(REF_SITE) not in sys.path:
        sys.path.insert(0, str(REF_SITE))
    return importlib.import_module("retrieve")


def _repoint():
    """The maintainer's one-line change: the "triton" backend's namespace is this library's."""
    _retrieve()
    itf = importlib.import_module("retrieve.interfaces")
    itf._OPS_NAMESPACE["triton"] = "retrieve_b200.ops"
    itf._OPS_LOADED.pop("triton", None)
    return itf


def _param_names(fn) -> list[str]:
    """Parameter names of a plain function, or of a registered custom op's schema."""
    op = getattr(fn, "_opoverload", None)
    if op is not None:
        return [a.name for a in op._schema.arguments]
    return list(inspect.signature(fn).parameters)


def test_every_op_the_modules_call_has_the_reference_signature():
    _retrieve()
    ref = importlib.import_module("retrieve.ops.reference")
    from retrieve_b200 import ops

    for name in OPS:
        want = _param_names(getattr(ref, name))
        got = _param_names(getattr(ops, name))
        assert got[: len(want)] == want, (name, want, got)


def test_repointed_namespace_resolves_to_this_library():
    itf = _repoint()
    from retrieve_b200 import ops

    assert itf.ops_for("triton") is ops
    from retrieve.modules.filters import ExactAttributeFilter

    f = ExactAttributeFilter(backend="triton")  # resolves the namespace at construction
    assert f.backend == "triton"


# --- GPU ---------------------------------------------------------------------------------------


def _attrs(n, c, a, card, g):
    x = torch.randint(0, card, (n, c, a), generator=g)
    x[torch.rand(n, c, a, generator=g) < 0.3] = -1  # -1 pads
    return x


def _queries_attrs(b, c, card, g):
    q = torch.randint(0, card, (b, c), generator=g)
    q[torch.rand(b, c, generator=g) < 0.5] = -1  # inactive clauses
    return q


def _recall(ids, ref_ids):
    hit = tot = 0
    for a, r in zip(ids.tolist(), ref_ids.tolist()):
        rs = {v for v in r if v >= 0}
        tot += len(rs)
        hit += len(rs & {v for v in a if v >= 0})
    return hit / max(tot, 1)


def _close_topk(ids, scores, ref_ids, ref_scores):
    """Float paths: recall@k >= 0.999 and |score| error <= 1e-2 relative, position by position."""
    assert _recall(ids.cpu(), ref_ids.cpu()) >= 0.999
    s, r = scores.cpu().float(), ref_scores.cpu().float()
    fin = torch.isfinite(r)
    assert torch.equal(fin, torch.isfinite(s))
    assert torch.all((s[fin] - r[fin]).abs() <= 1e-2 * r[fin].abs().clamp_min(1e-6))


@pytest.mark.gpu
def test_exact_attribute_filter_matches_the_torch_backend():
    _repoint()
    from retrieve.modules.filters import ExactAttributeFilter

    g = torch.Generator().manual_seed(11)
    n, c, a, b = 20_000, 4, 3, 16
    attrs = _attrs(n, c, a, 20, g).cuda()
    rev = torch.tensor([False, True, False, False]).cuda()
    qa = _queries_attrs(b, c, 20, g).cuda()
    scores = torch.randn(b, n, generator=g).cuda()
    mods = {}
    for backend in ("triton", "torch"):
        f = ExactAttributeFilter(backend=backend)
        f.register_index(attrs, clause_is_reverse=rev)
        mods[backend] = f
    ours, ref = mods["triton"], mods["torch"]
    assert torch.equal(ours.evaluate_mask(qa), ref.evaluate_mask(qa))
    assert torch.equal(ours.evaluate_mask(qa, 1000, 5000), ref.evaluate_mask(qa, 1000, 5000))
    assert torch.equal(ours.mask_scores(scores, qa), ref.mask_scores(scores, qa))
    (pi, pc), (ri, rc) = ours.evaluate_indices(qa), ref.evaluate_indices(qa)
    assert torch.equal(pc, rc)
    for row in range(b):
        assert torch.equal(pi[row, : pc[row]], ri[row, : rc[row]])


def _linr_pair(cls, k, filt, n=20_000, d=128, **kw):
    from retrieve.modules.filters import ExactAttributeFilter

    g = torch.Generator().manual_seed(12)
    items = torch.randn(n, d, generator=g)
    items = (items / items.norm(dim=1, keepdim=True)).cuda()
    attrs = _attrs(n, 4, 2, 8, g).cuda() if filt else None
    out = {}
    for backend in ("triton", "torch"):
        f = ExactAttributeFilter(backend=backend) if filt else None
        kwargs = dict(kw)
        if f is not None:
            kwargs["filter"] = f
        m = cls(k, backend=backend, **kwargs)
        m.register_index(items, attrs)
        out[backend] = m
    q = torch.randn(16, d, generator=g).cuda()
    qa = _queries_attrs(16, 4, 8, g).cuda() if filt else None
    return out["triton"], out["torch"], q, qa


@pytest.mark.gpu
@pytest.mark.parametrize("filt", [False, True])
def test_linr_v1_matches_the_torch_backend(filt):
    _repoint()
    from retrieve.modules.linr import LiNRV1

    ours, ref, q, qa = _linr_pair(LiNRV1, 50, filt)
    if filt:
        a = ours(q, ours.prepare_queries(qa))
        r = ref(q, ref.prepare_queries(qa))
    else:
        a, r = ours(q), ref(q)
    # the scores are cuBLAS's on both backends; the filter's masked scores are this library's
    assert torch.equal(a[1], r[1])
    assert _recall(a[0].cpu(), r[0].cpu()) == 1.0
    one = ours(q[:1]) if not filt else None  # B = 1: the GEMV path when it matches cuBLAS on this table
    if one is not None:
        _close_topk(*one, *ref(q[:1]))


@pytest.mark.gpu
def test_linr_v2_matches_the_torch_backend():
    _repoint()
    from retrieve.modules.linr import LiNRV2

    ours, ref, q, qa = _linr_pair(LiNRV2, 50, True)
    a = ours(q, ours.prepare_queries(qa))
    r = ref(q, ref.prepare_queries(qa))
    _close_topk(*a, *r)


@pytest.mark.gpu
def test_linr_v3_matches_the_torch_backend():
    _repoint()
    from retrieve.modules.linr import LiNRV3

    ours, ref, q, _ = _linr_pair(LiNRV3, 50, False)  # the reference's default pool (5000)
    assert ours.stage1.k == 5000
    _close_topk(*ours(q), *ref(q))


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["oporp", "simhash"])
def test_one_bit_knn_matches_the_torch_backend(kind):
    """Hamming scores are integers: the score rows equal bit for bit, and every returned id
    carries its own exact score (ties may order differently between the two top-k)."""
    _repoint()
    from retrieve.modules.bit_knn import OneBitKNN, SimHashKNN

    g = torch.Generator().manual_seed(13)
    n, d, k = 30_000, 128, 100
    items = torch.randn(n, d, generator=g).cuda()
    q = torch.randn(8, d, generator=g).cuda()
    mods = {}
    for backend in ("triton", "torch"):
        m = OneBitKNN(k, backend=backend) if kind == "oporp" else SimHashKNN(k, 256, backend=backend)
        m.register_index(items)
        mods[backend] = m
    ours, ref = mods["triton"], mods["torch"]
    assert torch.equal(ours.item_bits, ref.item_bits)
    (ai, asc), (ri, rsc) = ours(q), ref(q)
    assert torch.equal(asc, rsc)
    qbits = ours._project_query(q)
    pop = torch.zeros_like(ai, dtype=torch.float32)
    for row in range(q.shape[0]):
        x = qbits[row][None, :] ^ ours.item_bits[ai[row]]
        ham = sum(((x >> s) & 1).sum(dim=1) for s in range(64))
        pop[row] = (ours.d_total - 2 * ham).float()
    assert torch.equal(pop, asc)


def _silvertorch_loader():
    """What the maintainer's ``silvertorch.ops._load_ops`` becomes: importing it registers
    ``torch.ops.st.*`` from this library (the reference loader imports that module,
    retrieve/src/retrieve/ops/official/__init__.py:140-146)."""
    if "silvertorch.ops._load_ops" not in sys.modules:
        pkg = types.ModuleType("silvertorch")
        pkg.__path__ = []
        sub = types.ModuleType("silvertorch.ops")
        sub.__path__ = []
        load = types.ModuleType("silvertorch.ops._load_ops")
        importlib.import_module("retrieve_b200.st")
        sys.modules.update({"silvertorch": pkg, "silvertorch.ops": sub, "silvertorch.ops._load_ops": load})
    official = importlib.import_module("retrieve.ops.official")
    official._LOAD_MEMO.clear()
    return official.ensure_loaded()


@pytest.mark.gpu
@pytest.mark.parametrize("filter_mode", ["none", "exact"])
def test_silvertorch_module_on_this_library(filter_mode):
    _retrieve()
    st = _silvertorch_loader()
    assert st is torch.ops.st
    from oracle import ivf
    from retrieve.modules.silvertorch import SilverTorch

    g = torch.Generator().manual_seed(14)
    n, d, b, k = 20_000, 64, 8, 20
    items = torch.randn(n, d, generator=g)
    items = (items / items.norm(dim=1, keepdim=True)).cuda()
    q = torch.randn(b, d, generator=g).cuda()
    m = SilverTorch(k, n_lists=32, n_probe=4, filter_mode=filter_mode)
    if filter_mode == "exact":
        attrs = torch.randint(0, 6, (n, 3, 1), generator=g).cuda()
        m.register_index(items, item_clause_attrs=attrs)
        qa = torch.randint(0, 6, (b, 3), generator=g)
        qa[:, 1:] = -1
        prepared = m.prepare_queries(qa.cuda())
        ids, scores = m(q, prepared)
    else:
        m.register_index(items)
        ids, scores = m(q)
    probe = m._phase1_probe_ids(q)
    exact = None
    if filter_mode == "exact":  # the module's own exact layout and the prepared query attrs
        exact = (m.item_clause_attrs.cpu().numpy(), m.clause_slots.cpu().numpy(), m.clause_is_reverse.cpu().numpy(),
                 prepared.query_attrs.cpu().numpy())
    # the module's score path: the default OfficialConfig scores on the fp16 path
    cfg = m.official
    div = -1 if cfg.score_path == "int32" else (cfg.divisor or ivf.default_divisor(d))
    want_i, want_s = ivf.search(q.cpu().numpy(), probe.cpu().numpy(), m.cluster_offsets.cpu().numpy(),
                                m.cluster_sizes.cpu().numpy(), m.item_codes.cpu().numpy(),
                                m.sort_perm.cpu().numpy(), m.global_scale.reshape(-1).cpu().numpy(), k,
                                m._probe_width, divisor_for_int8=div, exact=exact)
    assert np.array_equal(scores.cpu().numpy(), want_s)
    assert np.array_equal(ids.cpu().numpy(), want_i)
