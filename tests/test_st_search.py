"""``st::search`` / ``st::probe_prep`` (retrieve_b200/st.py over rb_st_search /
rb_st_probe_prep) against the CPU restatement (oracle/ivf.py) and the fixture
the reference's own code produced (tests/golden/golden_ivf.npz).

CPU tests: the registered schemas equal the reference's pinned strings
(retrieve/tests/parity/test_official.py:65-116), the fake implementations give
the right shapes, and the C-ABI rejects bad arguments without a device. GPU
tests: bit-exact scores and ids against the oracle (whose ties follow the
reference scorer's slot order) and, up to ties, against the reference's fixture.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import ivf, knn
from retrieve_b200 import _lib
from tests.helpers import assert_topk_equal_up_to_ties

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "golden_ivf.npz")
N_CASES = len({k.split("_")[0] for k in GOLDEN.files})

PINNED_SEARCH = (
    "st::search(Tensor query, Tensor probe_ids, Tensor cluster_offsets, Tensor cluster_sizes, "
    "Tensor item_codes, Tensor sort_perm, Tensor global_scale, int k, "
    "int max_tensor_size_per_row, int divisor_for_int8=-1, Tensor? filtering_bit_mask=None, "
    "Tensor? bloom_index=None, Tensor? bloom_bundle_b_offsets=None, Tensor? plans=None, "
    "int plan_count=0, int max_stack_size=0, Tensor? query_plan_index=None, int bloom_k=0, "
    "int hash_k=0, Tensor? item_clause_attrs=None, Tensor? clause_slots=None, "
    "Tensor? clause_is_reverse=None, Tensor? query_clause_attrs=None) -> (Tensor, Tensor)"
)
PINNED_PROBE_PREP = (
    "st::probe_prep(Tensor query, Tensor probe_ids, Tensor cluster_offsets, Tensor cluster_sizes) "
    "-> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)"
)


def _st():
    import retrieve_b200.st  # noqa: F401  (registers the ops)

    return torch.ops.st


def _case(ci):
    p = f"c{ci}_"
    g = {k[len(p):]: GOLDEN[k] for k in GOLDEN.files if k.startswith(p)}
    n_lists, max_size, n_probe, d, k, b, width, div, ties = g["shape"].tolist()
    return g, dict(k=k, width=width, div=div, d=d, b=b)


# --- CPU -----------------------------------------------------------------------------------


PINNED_BLOOM_BUILD = (
    "st::bloom_index_build(Tensor feature_ids, Tensor feature_offsets, Tensor feature_values, "
    "float b_multiplier, int k, bool fast_build=False) -> (Tensor, Tensor)"
)


PINNED_FUSED = (
    "st::fused_kmean_ann(Tensor cluster_offsets, Tensor cluster_ids, Tensor cluster_length, Tensor embeddings, "
    "Tensor queries, int max_tensor_size_per_row, Tensor? filtering_bit_mask=None, int invalid_index_value=-1, "
    "int divisor_for_int8=-1, Tensor? filtering_bit_index=None, Tensor? per_embedding_scale=None) "
    "-> (Tensor, Tensor)"
)


def test_schemas_are_the_reference_ones():
    st = _st()
    assert str(st.search.default._schema) == PINNED_SEARCH
    assert str(st.probe_prep.default._schema) == PINNED_PROBE_PREP
    assert str(st.bloom_index_build.default._schema) == PINNED_BLOOM_BUILD
    # silvertorch/ops/csrc/fused_kmean_ann.cpp:401-414
    assert str(st.fused_kmean_ann.default._schema) == PINNED_FUSED


def test_fused_kmean_ann_fake_and_argument_errors():
    st = _st()
    from torch._subclasses.fake_tensor import FakeTensorMode

    from retrieve_b200 import st as rst

    with FakeTensorMode():
        raw, idx = st.fused_kmean_ann(torch.empty(9, dtype=torch.int64), torch.empty(4, 3, dtype=torch.int64),
                                      torch.empty(4, 3, dtype=torch.int64), torch.empty(100, 64, dtype=torch.int8),
                                      torch.empty(4, 64, dtype=torch.int8), 90)
        assert raw.shape == idx.shape == (4, 96) and raw.dtype == idx.dtype == torch.int32
        raw, _ = st.fused_kmean_ann(torch.empty(9, dtype=torch.int64), torch.empty(4, 3, dtype=torch.int64),
                                    torch.empty(4, 3, dtype=torch.int64), torch.empty(100, 64, dtype=torch.int8),
                                    torch.empty(4, 64, dtype=torch.int8), 90, divisor_for_int8=8)
        assert raw.dtype == torch.float16
        raw, _ = st.fused_kmean_ann(torch.empty(9, dtype=torch.int64), torch.empty(4, 3, dtype=torch.int64),
                                    torch.empty(4, 3, dtype=torch.int64), torch.empty(100, 64, dtype=torch.int8),
                                    torch.empty(4, 64, dtype=torch.int8), 90,
                                    per_embedding_scale=torch.empty(100, dtype=torch.float16))
        assert raw.dtype == torch.float16  # a per-doc divisor makes the raw scores fp16
    off, ids, lens = torch.tensor([0, 4]), torch.zeros(2, 1, dtype=torch.int64), torch.full((2, 1), 4)
    with pytest.raises(RuntimeError, match="dtype"):
        rst.fused_kmean_ann(off, ids, lens, torch.zeros(4, 64), torch.zeros(2, 64, dtype=torch.float16), 4)
    with pytest.raises(RuntimeError, match="scalar type"):
        rst.fused_kmean_ann(off, ids, lens, torch.zeros(4, 64, dtype=torch.float64), torch.zeros(2, 64), 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        rst.fused_kmean_ann(off, ids, lens, torch.zeros(4, 64, dtype=torch.int8), torch.zeros(2, 64, dtype=torch.int8),
                            4)


def test_fused_kmean_ann_capi_checks_need_no_device():
    lib = _lib.lib()
    n = ctypes.c_size_t(0)
    assert lib.rb_st_fused_kmean_ann_workspace_size(4, 8, 90, ctypes.byref(n)) == 0
    assert n.value >= 4 * 96 * 8
    assert lib.rb_st_fused_kmean_ann_workspace_size(-1, 8, 90, ctypes.byref(n)) == _lib.RB_ERR_INVALID_ARG

    fake = ctypes.c_void_p(16)  # never dereferenced: the checks fail first

    def call(b=4, d=64, p=8, width=90, div=-1, ws=None, ws_bytes=0, mask=None, mask_rows=4, index=None,
             dtype=_lib.RB_I8):
        return lib.rb_st_fused_kmean_ann(None, 8, None, None, p, None, 100, None, dtype, b, d, width, mask, mask_rows,
                                         2, index, None, -1, div, None, None, ws, ws_bytes, None)

    assert call(dtype=_lib.RB_E4M3) == _lib.RB_ERR_TYPE
    assert call(dtype=_lib.RB_F32, d=72) == _lib.RB_ERR_UNSUPPORTED  # 288 bytes: neither 256 nor 384 divides
    assert call(dtype=_lib.RB_F16, d=20) == _lib.RB_ERR_UNSUPPORTED  # not a multiple of 16 bytes
    assert call(dtype=_lib.RB_F32, d=96) == _lib.RB_ERR_WORKSPACE  # one 384-byte chain

    assert call(mask=fake, mask_rows=3) == _lib.RB_ERR_INVALID_ARG  # fewer mask rows than query rows
    assert call(mask=fake, mask_rows=3, index=fake) == _lib.RB_ERR_WORKSPACE  # rows picked by filtering_bit_index
    assert call(div=0) == _lib.RB_ERR_INVALID_ARG
    assert call(d=0) == _lib.RB_ERR_INVALID_ARG
    assert call(p=4096) == _lib.RB_ERR_UNSUPPORTED
    assert call(b=70000) == _lib.RB_ERR_UNSUPPORTED
    assert call() == _lib.RB_ERR_WORKSPACE
    assert call(b=0) == _lib.RB_OK and call(width=0) == _lib.RB_OK


def test_fake_shapes():
    st = _st()
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        q = torch.empty(4, 64)
        probe = torch.empty(4, 3, dtype=torch.int64)
        offsets = torch.empty(9, dtype=torch.int64)
        sizes = torch.empty(8, dtype=torch.int64)
        out = st.probe_prep(q, probe, offsets, sizes)
        assert [tuple(o.shape) for o in out] == [(4, 64), (4,), (4, 3), (4, 3), (4, 3), (12,), (4, 3), (12,), (12,)]
        assert [o.dtype for o in out[5:]] == [torch.int32] * 4
        ids, scores = st.search(q, probe, offsets, sizes, torch.empty(100, 64, dtype=torch.int8),
                                torch.empty(100, dtype=torch.int64), torch.empty(()), 7, 90)
        assert ids.shape == scores.shape == (4, 7) and ids.dtype == torch.int64


def test_cpu_tensors_raise():
    st = _st()
    with pytest.raises(RuntimeError):
        st.search(torch.zeros(2, 64), torch.zeros(2, 1, dtype=torch.int64), torch.tensor([0, 4]),
                  torch.tensor([4]), torch.zeros(4, 64, dtype=torch.int8), torch.arange(4), torch.tensor(1.0), 2, 4)


def test_argument_errors_raise_runtime_error():
    """The reference's TORCH_CHECKs raise RuntimeError (fork_search_cuda.cu:1280-1295); these
    fail before any device work (the CUDA implementation is called directly: CPU tensors
    would not dispatch to it)."""
    _st()
    from retrieve_b200 import st

    q = torch.zeros(2, 64)
    probe = torch.zeros(2, 1, dtype=torch.int64)
    off, sz = torch.tensor([0, 4]), torch.tensor([4])
    perm, gs = torch.arange(4), torch.tensor(1.0)
    with pytest.raises(RuntimeError, match="int8"):
        st.search(q, probe, off, sz, torch.zeros(4, 64, dtype=torch.float16), perm, gs, 2, 4)
    with pytest.raises(RuntimeError, match="D"):
        st.search(q, probe, off, sz, torch.zeros(4, 32, dtype=torch.int8), perm, gs, 2, 4)
    with pytest.raises(RuntimeError, match="one filter"):
        st.search(q, probe, off, sz, torch.zeros(4, 64, dtype=torch.int8), perm, gs, 2, 4,
                  filtering_bit_mask=torch.zeros(2, 1, dtype=torch.int64),
                  query_clause_attrs=torch.zeros(2, 1, dtype=torch.int32))
    with pytest.raises(RuntimeError, match="bloom"):
        st.search(q, probe, off, sz, torch.zeros(4, 64, dtype=torch.int8), perm, gs, 2, 4,
                  plans=torch.zeros(8, dtype=torch.int64))


def _adapter_positional(q, probe, off, sz, codes, perm, gs, mask=None, bloom=None, exact=None):
    """The 23 arguments in the order the reference's ``adapter.fork_search`` passes them, all
    positionally (retrieve/src/retrieve/ops/official/adapter.py:522-544); the dispatcher hands
    them to the registered CUDA impl the same way."""
    b = bloom
    return (q, probe, off, sz, codes, perm, gs, 2, 4, -1, mask,
            None if b is None else b[0], None if b is None else b[1], None if b is None else b[2],
            0 if b is None else 2, 0 if b is None else 4, None, 0 if b is None else 3, 0 if b is None else 7,
            *(exact if exact is not None else (None, None, None, None)))


@pytest.mark.parametrize("grouped", [False, True])
def test_search_binds_the_adapters_positional_call(grouped):
    """Every filter form passed positionally, as the dispatcher does, binds to the impl's
    parameters and reaches its argument checks (no TypeError)."""
    _st()
    from retrieve_b200 import st

    fn = st.search_grouped if grouped else st.search_rows
    q = torch.zeros(2, 64)
    probe = torch.zeros(2, 1, dtype=torch.int64)
    off, sz = torch.tensor([0, 4]), torch.tensor([4])
    perm, gs = torch.arange(4), torch.tensor(1.0)
    codes = torch.zeros(4, 64, dtype=torch.int8)
    mask = torch.zeros(2, 1, dtype=torch.int64)
    exact = (torch.zeros(1, 4, dtype=torch.int32), torch.tensor([0, 1]), torch.tensor([False]),
             torch.zeros(2, 1, dtype=torch.int32))
    bloom = (torch.zeros(64, dtype=torch.int64), torch.tensor([0, 2]), torch.zeros(16, dtype=torch.int64))
    args = _adapter_positional(q, probe, off, sz, codes, perm, gs, mask=mask, exact=exact)
    assert len(args) == 23
    with pytest.raises(RuntimeError, match="one filter"):
        fn(*args)
    # each filter alone binds and fails later, on the CPU tensors (the impl serves CUDA)
    for kw in ({"mask": mask}, {"exact": exact}, {"bloom": bloom}, {"bloom": bloom, "exact": exact}):
        with pytest.raises(RuntimeError, match="CUDA|device"):
            fn(*_adapter_positional(q, probe, off, sz, codes, perm, gs, **kw))


REF_CPU_LIB = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "silvertorch_ref_cpu.so"


@pytest.mark.skipif(not REF_CPU_LIB.exists(), reason="the reference's CPU st ops are not built here")
def test_registers_beside_the_reference_cpu_ops():
    """The drop-in layout: the reference's CPU build defines the st:: schemas and
    its CPU ops; importing retrieve_b200.st then adds the CUDA kernels (search,
    probe_prep, fused_kmean_ann, ...). Run in a child process (one registry per process)."""
    import subprocess
    import sys

    code = (
        "import torch\n"
        f"torch.ops.load_library({str(REF_CPU_LIB)!r})\n"
        "import retrieve_b200.st\n"
        "has = torch._C._dispatch_has_kernel_for_dispatch_key\n"
        "assert has('st::search', 'CUDA') and has('st::probe_prep', 'CUDA')\n"
        "assert has('st::fused_kmean_ann', 'CPU') and has('st::fused_kmean_ann', 'CUDA')\n"
    )
    root = Path(__file__).resolve().parent.parent
    r = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]


def test_capi_argument_checks_need_no_device():
    lib = _lib.lib()
    n = ctypes.c_size_t(0)
    assert lib.rb_st_search_workspace_size(16, 128, 8, 32, 700, ctypes.byref(n)) == 0
    # codes + scales + positions [16, 704] int64 + counts + winners, at least
    assert n.value >= 16 * 704 * 8
    assert lib.rb_st_search_workspace_size(16, 128, 8, 0, 700, ctypes.byref(n)) == _lib.RB_ERR_INVALID_ARG

    def call(b=4, d=128, p=8, k=10, width=256, div=-1, ws=None, ws_bytes=0, mask=None, qattrs=None, attrs=None,
             docs=1000, bloom=None, bloom_k=5, stack=3, plan_words=64):
        f = _lib.StFilter(filtering_bit_mask=mask, item_clause_attrs=attrs, attr_rows=3, attr_docs=docs,
                          clause_slots=attrs, clause_is_reverse=attrs, query_clause_attrs=qattrs, n_clauses=2,
                          bloom_index=bloom, bloom_words=100, bundle_b_offsets=bloom, n_bundles=1, plans=bloom,
                          plan_words=plan_words, plan_count=4, max_stack_size=stack, bloom_k=bloom_k, hash_k=7)
        return lib.rb_st_search(None, b, d, None, p, None, None, 16, None, 1000, None, None, k, width, div,
                                ctypes.byref(f), None, None, ws, ws_bytes, None)

    assert call(d=2048) == _lib.RB_ERR_UNSUPPORTED  # D > 1024
    assert call(p=4096) == _lib.RB_ERR_UNSUPPORTED  # more than 2048 probes
    assert call(k=2000, width=2048) == _lib.RB_ERR_UNSUPPORTED  # min(k, width) > 1024
    assert call(k=300, width=200) == _lib.RB_ERR_WORKSPACE  # min(300, 224) fits; then the workspace check
    assert call(k=1000, width=2048) == _lib.RB_ERR_WORKSPACE  # large k: the 1280-entry lists
    assert call(div=0) == _lib.RB_ERR_INVALID_ARG
    assert call(b=-1) == _lib.RB_ERR_INVALID_ARG
    assert call(b=70000) == _lib.RB_ERR_UNSUPPORTED
    assert call() == _lib.RB_ERR_WORKSPACE
    assert b"workspace" in lib.rb_last_error()
    fake = ctypes.c_void_p(16)  # never dereferenced: the checks fail first
    assert call(mask=fake, qattrs=fake, attrs=fake) == _lib.RB_ERR_INVALID_ARG  # one filter only
    assert call(qattrs=fake) == _lib.RB_ERR_INVALID_ARG  # exact filter without its tables
    assert call(qattrs=fake, attrs=fake, docs=999) == _lib.RB_ERR_INVALID_ARG  # attrs narrower than N
    assert call(qattrs=fake, attrs=fake) == _lib.RB_ERR_WORKSPACE
    assert call(bloom=fake) == _lib.RB_ERR_WORKSPACE  # a well-formed bloom filter
    assert call(bloom=fake, qattrs=fake, attrs=fake) == _lib.RB_ERR_INVALID_ARG  # one filter only
    assert call(bloom=fake, bloom_k=11) == _lib.RB_ERR_UNSUPPORTED  # more positions than SilverTorch resolves
    assert call(bloom=fake, stack=17) == _lib.RB_ERR_UNSUPPORTED  # deeper plans than the device stack
    assert call(bloom=fake, plan_words=16) == _lib.RB_ERR_INVALID_ARG  # 4 plan slots need 32 header words
    assert call(b=0) == _lib.RB_OK  # nothing to do: no device touched


# --- GPU -----------------------------------------------------------------------------------


def _run(st, g, meta, **kw):
    dev = "cuda"
    t = {k: torch.from_numpy(np.ascontiguousarray(g[k])).to(dev)
         for k in ("query", "probe", "offsets", "sizes", "codes", "sort_perm")}
    gs = torch.from_numpy(g["gs"]).to(dev)
    ids, scores = st.search(t["query"], t["probe"], t["offsets"], t["sizes"], t["codes"], t["sort_perm"], gs,
                            meta["k"], meta["width"], **kw)
    return ids.cpu().numpy(), scores.cpu().numpy()


def _assert_exact(ids, scores, ref_ids, ref_scores):
    assert np.array_equal(scores, ref_scores), f"{int((scores != ref_scores).sum())} score slots differ"
    assert np.array_equal(ids, ref_ids), f"{int((ids != ref_ids).sum())} id slots differ"


@pytest.mark.gpu
@pytest.mark.parametrize("ci", range(N_CASES))
def test_search_int32_path(ci):
    st = _st()
    g, meta = _case(ci)
    ids, scores = _run(st, g, meta)
    want = ivf.search(g["query"], g["probe"], g["offsets"], g["sizes"], g["codes"], g["sort_perm"], g["gs"],
                      meta["k"], meta["width"])
    _assert_exact(ids, scores, *want)
    assert_topk_equal_up_to_ties(ids, scores, g["ids32"], g["sc32"])


@pytest.mark.gpu
@pytest.mark.parametrize("ci", range(N_CASES))
def test_search_fp16_path(ci):
    st = _st()
    g, meta = _case(ci)
    ids, scores = _run(st, g, meta, divisor_for_int8=meta["div"])
    want = ivf.search(g["query"], g["probe"], g["offsets"], g["sizes"], g["codes"], g["sort_perm"], g["gs"],
                      meta["k"], meta["width"], divisor_for_int8=meta["div"])
    _assert_exact(ids, scores, *want)
    assert_topk_equal_up_to_ties(ids, scores, g["ids16"], g["sc16"])


@pytest.mark.gpu
@pytest.mark.parametrize("ci", range(N_CASES))
def test_search_filter_mask(ci):
    st = _st()
    g, meta = _case(ci)
    words = ivf.pack_mask_high_first(g["mask"])
    ids, scores = _run(st, g, meta, filtering_bit_mask=torch.from_numpy(words).cuda())
    want = ivf.search(g["query"], g["probe"], g["offsets"], g["sizes"], g["codes"], g["sort_perm"], g["gs"],
                      meta["k"], meta["width"], filtering_bit_mask=words)
    _assert_exact(ids, scores, *want)
    assert_topk_equal_up_to_ties(ids, scores, g["idsm"], g["scm"])


def _exact_inputs(rng, n, b, c=3, a_max=3, n_vocab=6, reverse=(True, False, False)):
    """Small-vocabulary attrs (a high pass rate), about 20 % of query clauses inactive,
    clause 0 reversed; the layout of the exact filter."""
    attrs = rng.integers(-1, n_vocab, (n, c, a_max))
    q = rng.integers(0, n_vocab, (b, c))
    q[rng.random((b, c)) < 0.2] = -1
    rev = np.array(reverse[:c], dtype=bool)
    slots, clause_slots = ivf.exact_layout(attrs)
    return attrs, rev, q, slots, clause_slots, ivf.exact_query(q)


@pytest.mark.gpu
@pytest.mark.parametrize("ci", range(N_CASES))
@pytest.mark.parametrize("score_path", ["int32", "fp16"])
def test_search_exact_clause_filter(ci, score_path):
    """The layer's exact path: the clauses tested inside st::search equal the oracle
    bit for bit, and the same predicate given as a full-N mask; bloom plans with the
    exact recheck give the same result."""
    st = _st()
    g, meta = _case(ci)
    rng = np.random.default_rng(ci)
    n = g["codes"].shape[0]
    attrs, rev, q, slots, clause_slots, qq = _exact_inputs(rng, n, meta["b"])
    div = -1 if score_path == "int32" else meta["div"]
    ex = (torch.from_numpy(slots).cuda(), torch.from_numpy(clause_slots).cuda(), torch.from_numpy(rev).cuda(),
          torch.from_numpy(qq).cuda())
    ids, scores = _run(st, g, meta, divisor_for_int8=div, item_clause_attrs=ex[0], clause_slots=ex[1],
                       clause_is_reverse=ex[2], query_clause_attrs=ex[3])
    args = (g["query"], g["probe"], g["offsets"], g["sizes"], g["codes"], g["sort_perm"], g["gs"], meta["k"],
            meta["width"])
    want = ivf.search(*args, divisor_for_int8=div, exact=(slots, clause_slots, rev, qq))
    _assert_exact(ids, scores, *want)
    from oracle import filters

    words = ivf.pack_mask_high_first(filters.clause_mask(attrs, rev, q))
    _assert_exact(ids, scores, *ivf.search(*args, divisor_for_int8=div, filtering_bit_mask=words))
    ids2, scores2 = _run(st, g, meta, divisor_for_int8=div, item_clause_attrs=ex[0], clause_slots=ex[1],
                         clause_is_reverse=ex[2], query_clause_attrs=ex[3],
                         plans=torch.zeros(8, dtype=torch.uint8, device="cuda"), plan_count=1)
    _assert_exact(ids2, scores2, ids, scores)


def _layout(rng, n_lists, max_size, d, b, p):
    sizes = rng.integers(0, max_size + 1, n_lists).astype(np.int64)
    offsets = np.r_[0, np.cumsum(sizes)].astype(np.int64)
    n = int(offsets[-1])
    codes = rng.integers(-128, 128, (n, d)).astype(np.int8)
    perm = rng.permutation(n).astype(np.int64)
    probe = np.argsort(rng.random((b, n_lists)), axis=1)[:, :p].astype(np.int64)
    q = rng.standard_normal((b, d)).astype(np.float32)
    width = int(sizes[probe].sum(1).max())
    return q, probe, offsets, sizes, codes, perm, width


@pytest.mark.gpu
@pytest.mark.parametrize("k", [1, 100, 224, 225, 1000])
def test_search_wide_rows_and_edge_shapes(k):
    """Wide rows (many warps of candidates per list), D not a multiple of 16 (scalar
    dot), empty clusters, k above the probed count (pads), and ties from repeated
    code rows."""
    st = _st()
    rng = np.random.default_rng(k)
    for d, n_lists, max_size, b, p in ((128, 64, 600, 8, 32), (100, 32, 90, 5, 8), (64, 16, 40, 3, 2)):
        q, probe, offsets, sizes, codes, perm, width = _layout(rng, n_lists, max_size, d, b, p)
        codes[1::3] = codes[0]  # many equal dots
        gs = np.float32(0.0123)
        t = [torch.from_numpy(x).cuda() for x in (q, probe, offsets, sizes, codes, perm)]
        ids, scores = st.search(*t, torch.tensor(gs).cuda(), k, width)
        want = ivf.search(q, probe, offsets, sizes, codes, perm, gs, k, width)
        _assert_exact(ids.cpu().numpy(), scores.cpu().numpy(), *want)


@pytest.mark.gpu
def test_search_zero_probes_and_zero_width():
    st = _st()
    q = torch.randn(3, 64, device="cuda")
    offsets = torch.tensor([0, 10], device="cuda")
    sizes = torch.tensor([10], device="cuda")
    codes = torch.ones(10, 64, dtype=torch.int8, device="cuda")
    perm = torch.arange(10, device="cuda")
    gs = torch.tensor(1.0, device="cuda")
    for probe, width in ((torch.zeros(3, 0, dtype=torch.int64, device="cuda"), 10),
                         (torch.zeros(3, 1, dtype=torch.int64, device="cuda"), 0)):
        ids, scores = st.search(q, probe, offsets, sizes, codes, perm, gs, 5, width)
        assert (ids == -1).all() and torch.isneginf(scores).all()


@pytest.mark.gpu
@pytest.mark.parametrize("d", [128, 192, 768])
def test_probe_prep_matches_oracle(d):
    """The layout the reference checks (retrieve/tests/parity/test_official.py:676-697),
    with its edge rows (zeros, a tiny value, exact half-code quotients)."""
    st = _st()
    rng = np.random.default_rng(9)
    q = rng.standard_normal((2000, d)).astype(np.float32)
    q[0] = 0.0
    q[1] = 0.0
    q[1, 3] = 1e-30
    q[2] = (np.arange(d) % 3 - 1.0).astype(np.float32)
    q[2, 0] = 2.54
    q[2, 1:5] = [0.01, -0.01, 1.27, -1.27]
    sizes = rng.integers(0, 150, 300).astype(np.int64)
    offsets = np.r_[0, np.cumsum(sizes)].astype(np.int64)
    probe = np.argsort(rng.random((2000, 300)), axis=1)[:, :24].astype(np.int64)
    out = st.probe_prep(*(torch.from_numpy(x).cuda() for x in (q, probe, offsets, sizes)))
    want = ivf.probe_prep(q, probe, offsets, sizes)
    for got, ref in zip(out, want, strict=True):
        got = got.cpu().numpy()
        assert got.shape == np.shape(ref) and np.array_equal(got, ref)
    codes, scales = knn.quantize_int8(q)
    assert np.array_equal(out[1].cpu().numpy(), scales)


# --- the grouped scorer (rb_st_search_grouped) -----------------------------------------------


def test_grouped_capi_checks_need_no_device():
    lib = _lib.lib()
    n = ctypes.c_size_t(0)
    assert lib.rb_st_search_grouped_workspace_size(16, 128, 8, 1024, 32, 700, ctypes.byref(n)) == 0
    assert n.value >= 16 * 8 * 256 * 8  # one 256-entry list per (row, probe)

    def call(p=8, ws=None, ws_bytes=0):
        return lib.rb_st_search_grouped(None, 4, 128, None, p, None, None, 16, None, 1000, None, None, 10, 256, -1,
                                        None, None, None, ws, ws_bytes, None)

    assert call(p=1500) == _lib.RB_ERR_UNSUPPORTED  # more than 1024 probes a row
    assert call() == _lib.RB_ERR_WORKSPACE


def _grouped(g, meta, **kw):
    _st()
    from retrieve_b200 import st

    t = {k: torch.from_numpy(np.ascontiguousarray(g[k])).cuda()
         for k in ("query", "probe", "offsets", "sizes", "codes", "sort_perm")}
    ids, scores = st.search_grouped(t["query"], t["probe"], t["offsets"], t["sizes"], t["codes"], t["sort_perm"],
                                    torch.from_numpy(g["gs"]).cuda(), meta["k"], meta["width"], **kw)
    return ids.cpu().numpy(), scores.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("ci", range(N_CASES))
def test_grouped_equals_the_row_path_and_the_oracle(ci):
    """Int32 and fp16 paths, the full-N mask and the exact clauses: bit for bit the
    oracle (ties to the reference scorer's lower slot), hence the row path."""
    g, meta = _case(ci)
    args = (g["query"], g["probe"], g["offsets"], g["sizes"], g["codes"], g["sort_perm"], g["gs"], meta["k"],
            meta["width"])
    _assert_exact(*_grouped(g, meta), *ivf.search(*args))
    _assert_exact(*_grouped(g, meta, divisor_for_int8=meta["div"]), *ivf.search(*args, divisor_for_int8=meta["div"]))
    words = ivf.pack_mask_high_first(g["mask"])
    _assert_exact(*_grouped(g, meta, filtering_bit_mask=torch.from_numpy(words).cuda()),
                  *ivf.search(*args, filtering_bit_mask=words))
    rng = np.random.default_rng(ci)
    _, rev, _, slots, clause_slots, qq = _exact_inputs(rng, g["codes"].shape[0], meta["b"])
    got = _grouped(g, meta, item_clause_attrs=torch.from_numpy(slots).cuda(),
                   clause_slots=torch.from_numpy(clause_slots).cuda(), clause_is_reverse=torch.from_numpy(rev).cuda(),
                   query_clause_attrs=torch.from_numpy(qq).cuda())
    _assert_exact(*got, *ivf.search(*args, exact=(slots, clause_slots, rev, qq)))


@pytest.mark.gpu
@pytest.mark.parametrize("k", [1, 100, 224, 225, 1000])
def test_grouped_many_rows_per_cluster(k):
    """More probing rows per cluster than one task holds (several tasks per cluster),
    wide rows, D = 100 (the unaligned staging), D = 1024 (the largest tile) and ties."""
    _st()
    from retrieve_b200 import st

    rng = np.random.default_rng(100 + k)
    for d, n_lists, max_size, b, p in ((128, 8, 500, 200, 4), (100, 32, 90, 37, 8), (1024, 16, 70, 20, 3)):
        q, probe, offsets, sizes, codes, perm, width = _layout(rng, n_lists, max_size, d, b, p)
        codes[1::3] = codes[0]
        gs = np.float32(0.0123)
        t = [torch.from_numpy(x).cuda() for x in (q, probe, offsets, sizes, codes, perm)]
        ids, scores = st.search_grouped(*t, torch.tensor(gs).cuda(), k, width)
        _assert_exact(ids.cpu().numpy(), scores.cpu().numpy(), *ivf.search(q, probe, offsets, sizes, codes, perm, gs,
                                                                          k, width))


# --- SilverTorch's bloom filter (plans without the exact recheck) -------------------------------

BLOOM = np.load(Path(__file__).resolve().parent / "golden" / "golden_bloom_st.npz")


@pytest.mark.gpu
@pytest.mark.parametrize("grouped", [False, True])
@pytest.mark.parametrize("plan_index", [False, True])
def test_search_bloom_plans(grouped, plan_index):
    """The reference's own bloom index, parsed plans and CPU search (the fixture): the op
    with the prepared plan blob returns the oracle's search under the reference's bloom
    mask, bit for bit (false positives included), row by row or through query_plan_index."""
    _st()
    from retrieve_b200 import st

    n = int(BLOOM["n"])
    want_mask = np.unpackbits(BLOOM["mask_bits"], axis=1)[:, :n].astype(bool)
    n_plans = want_mask.shape[0]
    rng = np.random.default_rng(3)
    b = 2 * n_plans if plan_index else n_plans
    cuts = np.sort(rng.integers(0, n + 1, 59))
    sizes = np.diff(np.r_[0, cuts, n]).astype(np.int64)  # 60 clusters covering the n docs
    offsets = np.r_[0, np.cumsum(sizes)].astype(np.int64)
    d = 64
    codes = rng.integers(-128, 128, (n, d)).astype(np.int8)
    perm = rng.permutation(n).astype(np.int64)
    probe = np.argsort(rng.random((b, len(sizes))), axis=1)[:, :12].astype(np.int64)
    q = rng.standard_normal((b, d)).astype(np.float32)
    width = int(sizes[probe].sum(1).max())
    rows = np.arange(b) % n_plans if plan_index else np.arange(b)
    blob = ivf.plan_blob(BLOOM["plan_data"], BLOOM["plan_offsets"], n_plans)
    t = [torch.from_numpy(x).cuda() for x in (q, probe, offsets, sizes, codes, perm)]
    fn = st.search_grouped if grouped else st.search_rows
    ids, scores = fn(*t, torch.tensor(0.02).cuda(), 50, width,
                     bloom_index=torch.from_numpy(BLOOM["bloom_index"]).cuda(),
                     bloom_bundle_b_offsets=torch.from_numpy(BLOOM["bundle_b_offsets"]).cuda(),
                     plans=torch.from_numpy(blob).cuda(), plan_count=n_plans,
                     max_stack_size=int(BLOOM["max_stack"]),
                     query_plan_index=torch.from_numpy(rows.astype(np.int64)).cuda() if plan_index else None,
                     bloom_k=int(BLOOM["k"]), hash_k=int(BLOOM["hash_k"]))
    words = ivf.pack_mask_high_first(want_mask[rows])
    want = ivf.search(q, probe, offsets, sizes, codes, perm, np.float32(0.02), 50, width, filtering_bit_mask=words)
    _assert_exact(ids.cpu().numpy(), scores.cpu().numpy(), *want)


@pytest.mark.gpu
@pytest.mark.parametrize("ci", range(N_CASES))
def test_registered_op_equals_the_row_scorer_for_every_filter(ci):
    """torch.ops.st.search picks its scorer (grouped unless bloom plans come without the exact
    recheck, or more than 1024 probes a row): through the dispatcher, with all 23 arguments
    positional as the reference's adapter passes them, it equals the row scorer bit for bit
    unfiltered, with a full-N mask and with the exact clauses."""
    _st()
    from retrieve_b200 import st

    g, meta = _case(ci)
    t = [torch.from_numpy(np.ascontiguousarray(g[key])).cuda()
         for key in ("query", "probe", "offsets", "sizes", "codes", "sort_perm")]
    gs = torch.from_numpy(g["gs"]).cuda()
    k, width, div = meta["k"], meta["width"], meta["div"]
    n, b = g["codes"].shape[0], meta["b"]
    rng = np.random.default_rng(100 + ci)
    mask = torch.from_numpy(ivf.pack_mask_high_first(rng.random((b, n)) < 0.6)).cuda()
    _, rev, _, slots_t, clause_slots, qq = _exact_inputs(rng, n, b)
    exact = (torch.from_numpy(slots_t).cuda(), torch.from_numpy(clause_slots).cuda(), torch.from_numpy(rev).cuda(),
             torch.from_numpy(qq).cuda())
    for m, ex in ((None, None), (mask, None), (None, exact)):
        args = (*t, gs, k, width, div, m, None, None, None, 0, 0, None, 0, 0,
                *(ex if ex is not None else (None, None, None, None)))
        got = torch.ops.st.search(*args)
        want = st.search_rows(*args)
        assert torch.equal(got[0], want[0]) and torch.equal(got[1], want[1])


@pytest.mark.gpu
@pytest.mark.parametrize("d,k", [(128, 100), (256, 10), (512, 100), (128, 300), (128, 1)])
def test_grouped_tensor_core_scan_equals_the_row_scorer(d, k):
    """The grouped scorer's tensor-core form (int8 rows of 128 / 256 / 512 bytes, no bloom plans):
    ragged and empty clusters, more than 128 rows probing one cluster, fp16 and int32 raw scores,
    unfiltered, full-N mask and exact clauses: bit for bit the row scorer and the oracle; and a
    width that cuts rows, against the row scorer."""
    _st()
    from retrieve_b200 import st

    rng = np.random.default_rng(d + k)
    n_lists, b, p = 40, 300, 6
    sizes = rng.integers(0, 700, n_lists).astype(np.int64)
    sizes[3] = 0
    sizes[7] = 2500
    offsets = np.r_[0, np.cumsum(sizes)].astype(np.int64)
    n = int(offsets[-1])
    codes = rng.integers(-128, 128, (n, d)).astype(np.int8)
    codes[: n // 3, : d // 2] = 1  # ties among many rows
    perm = rng.permutation(n).astype(np.int64)
    probe = np.argsort(rng.random((b, n_lists)), axis=1)[:, :p].astype(np.int64)
    probe[:150, 0] = 7  # 150 rows probe the long cluster: two tasks of it
    q = rng.standard_normal((b, d)).astype(np.float32)
    width = 8192  # every row's probed total fits (the oracle's requirement)
    gs = np.float32(0.013)
    t = [torch.from_numpy(x).cuda() for x in (q, probe, offsets, sizes, codes, perm)]
    mask = ivf.pack_mask_high_first(rng.random((b, n)) < 0.7)
    _, rev, _, slots_t, clause_slots, qq = _exact_inputs(rng, n, b)
    exact = dict(item_clause_attrs=torch.from_numpy(slots_t).cuda(), clause_slots=torch.from_numpy(clause_slots).cuda(),
                 clause_is_reverse=torch.from_numpy(rev).cuda(), query_clause_attrs=torch.from_numpy(qq).cuda())
    for div in (-1, ivf.default_divisor(d)):
        for flt in ({}, {"filtering_bit_mask": torch.from_numpy(mask).cuda()}, exact):
            got = st.search_grouped(*t, torch.tensor(gs).cuda(), k, width, div, **flt)
            rows = st.search_rows(*t, torch.tensor(gs).cuda(), k, width, div, **flt)
            assert torch.equal(got[0], rows[0]) and torch.equal(got[1], rows[1])
            ex = (slots_t, clause_slots, rev, qq) if "item_clause_attrs" in flt else None
            want = ivf.search(q, probe, offsets, sizes, codes, perm, gs, k, width, div,
                              filtering_bit_mask=mask if "filtering_bit_mask" in flt else None, exact=ex)
            _assert_exact(got[0].cpu().numpy(), got[1].cpu().numpy(), *want)
    got = st.search_grouped(*t, torch.tensor(gs).cuda(), k, 1024)
    rows = st.search_rows(*t, torch.tensor(gs).cuda(), k, 1024)
    assert torch.equal(got[0], rows[0]) and torch.equal(got[1], rows[1])


@pytest.mark.gpu
def test_bloom_index_build_on_device():
    """st::bloom_index_build on the device equals the reference's CPU builder bit for bit;
    the fixed width (st::bloom_index_build_fixed, CUDA only in the reference) equals the
    oracle's restatement, and plans searched over it equal the oracle's plan masks."""
    st = _st()
    fid, off, val = ivf.attrs_to_features(BLOOM["attrs"])
    t = [torch.from_numpy(x).cuda() for x in (fid, off, val)]
    index, boff = st.bloom_index_build(*t, 10.0, int(BLOOM["k"]))
    assert np.array_equal(boff.cpu().numpy(), BLOOM["bundle_b_offsets"])
    assert np.array_equal(index.cpu().numpy(), BLOOM["bloom_index"])
    for bits in (64, 257):
        index_f, boff_f = st.bloom_index_build_fixed(*t, bits, int(BLOOM["k"]))
        want_i, want_b = ivf.bloom_index_build(fid, off, val, 2.0, int(BLOOM["k"]), bits_per_doc=bits)
        assert np.array_equal(boff_f.cpu().numpy(), want_b) and np.array_equal(index_f.cpu().numpy(), want_i)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("ci", [0, 3, 6])
def test_sharded_search_on_one_gpu(world, ci):
    """The row-sharded search's three steps on one GPU (the shards called in turn): the
    [W, B, k'] pairs of rb_st_search_shard, rb_merge_pairs and rb_st_search_finish equal
    the single-table st::search bit for bit, ties included, unfiltered and with the exact
    clauses (whole-table filter tables on every shard)."""
    _st()
    from retrieve_b200 import ops, st
    from retrieve_b200.shard import ivf_shard_bounds

    g, meta = _case(ci)
    t = {key: torch.from_numpy(np.ascontiguousarray(g[key])).cuda()
         for key in ("query", "probe", "offsets", "sizes", "codes", "sort_perm")}
    gs = torch.from_numpy(g["gs"]).cuda()
    k, width = meta["k"], meta["width"]
    rng = np.random.default_rng(ci)
    _, rev, _, slots_t, clause_slots, qq = _exact_inputs(rng, g["codes"].shape[0], meta["b"])
    exact = dict(item_clause_attrs=torch.from_numpy(slots_t).cuda(),
                 clause_slots=torch.from_numpy(clause_slots).cuda(), clause_is_reverse=torch.from_numpy(rev).cuda(),
                 query_clause_attrs=torch.from_numpy(qq).cuda())
    for filters in ({}, exact):
        want = torch.ops.st.search(t["query"], t["probe"], t["offsets"], t["sizes"], t["codes"], t["sort_perm"], gs,
                                   k, width, **filters)
        pairs = []
        for r in range(world):
            _, _, lo, hi = ivf_shard_bounds(g["offsets"], world, r)
            pairs.append(st.search_shard(t["query"], t["probe"], t["offsets"], t["sizes"], g["codes"].shape[0], lo,
                                         t["codes"][lo:hi], k, width, **filters))
        stack = torch.stack(pairs).contiguous()
        slots, raw = ops.merge_pairs(stack, stack.shape[2])
        ids, scores = st.search_finish(t["query"], t["probe"], t["offsets"], t["sizes"], t["sort_perm"], gs, k,
                                       width, slots, raw)
        _assert_exact(ids.cpu().numpy(), scores.cpu().numpy(), want[0].cpu().numpy(), want[1].cpu().numpy())


def _fused_inputs(g):
    codes, _ = knn.quantize_int8(g["query"])
    lengths = g["sizes"][g["probe"]]
    t = dict(offsets=g["offsets"], ids=g["probe"], lengths=lengths, codes=g["codes"], q=codes)
    return {key: torch.from_numpy(np.ascontiguousarray(v)).cuda() for key, v in t.items()}, codes, lengths


@pytest.mark.gpu
@pytest.mark.parametrize("ci", range(N_CASES))
def test_fused_kmean_ann_rows(ci):
    """st::fused_kmean_ann on int8 codes: the int32 and fp16 rows equal the restatement's bit
    for bit (slot order, pads, invalid_index_value), with and without a full-N mask, and hold
    the reference CPU scorer's (position, dot) multiset per row."""
    st = _st()
    g, meta = _case(ci)
    t, codes, lengths = _fused_inputs(g)
    width = meta["width"]
    raw, idx = st.fused_kmean_ann(t["offsets"], t["ids"], t["lengths"], t["codes"], t["q"], width)
    want_r, want_i = ivf.fused_kmean_ann(codes, g["offsets"], g["probe"], lengths, g["codes"], width)
    assert raw.dtype == torch.int32 and idx.dtype == torch.int32
    assert np.array_equal(raw.cpu().numpy(), want_r) and np.array_equal(idx.cpu().numpy(), want_i)
    for r in range(meta["b"]):
        valid = g["idx"][r] >= 0
        got = idx.cpu().numpy()[r]
        assert sorted(zip(got[got >= 0].tolist(), raw.cpu().numpy()[r][got >= 0].tolist())) == sorted(
            zip(g["idx"][r][valid].tolist(), g["raw"][r][valid].tolist()))
    words = ivf.pack_mask_high_first(g["mask"])
    r16, i16 = st.fused_kmean_ann(t["offsets"], t["ids"], t["lengths"], t["codes"], t["q"], width,
                                  filtering_bit_mask=torch.from_numpy(words).cuda(), invalid_index_value=-3,
                                  divisor_for_int8=meta["div"])
    w16, wi16 = ivf.fused_kmean_ann(codes, g["offsets"], g["probe"], lengths, g["codes"], width,
                                    divisor_for_int8=meta["div"], filtering_bit_mask=words, invalid_index_value=-3)
    assert r16.dtype == torch.float16
    assert np.array_equal(r16.cpu().numpy().view(np.uint16), w16.view(np.uint16))
    assert np.array_equal(i16.cpu().numpy(), wi16)


@pytest.mark.gpu
def test_fused_kmean_ann_lengths_and_clipping():
    """Per-(row, probe) lengths shorter than the clusters, zero and negative lengths, a
    cluster longer than the row, repeated probes and a row width that is not a multiple of 32."""
    st = _st()
    rng = np.random.default_rng(11)
    sizes = rng.integers(0, 150, 40)
    offsets = np.r_[0, np.cumsum(sizes)].astype(np.int64)
    n, d, b, p = int(offsets[-1]), 96, 24, 6
    codes = rng.integers(-127, 128, (n, d), dtype=np.int8)
    q = rng.integers(-127, 128, (b, d), dtype=np.int8)
    probe = rng.integers(0, 40, (b, p)).astype(np.int64)
    probe[0, :3] = 7  # repeated probes
    lengths = np.minimum(sizes[probe], rng.integers(-5, 150, (b, p))).astype(np.int64)
    for width in (100, 160, 700):
        dev = [torch.from_numpy(np.ascontiguousarray(v)).cuda() for v in (offsets, probe, lengths, codes, q)]
        raw, idx = st.fused_kmean_ann(*dev, width)
        want_r, want_i = ivf.fused_kmean_ann(q, offsets, probe, lengths, codes, width)
        assert np.array_equal(raw.cpu().numpy(), want_r) and np.array_equal(idx.cpu().numpy(), want_i)


FUSED = np.load(Path(__file__).resolve().parent / "golden" / "golden_fused.npz")


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["scaled", "scaled_div", "index_i32", "index_scaled"])
def test_fused_kmean_ann_scale_and_mask_rows(case):
    """per_embedding_scale and filtering_bit_index on the device: bit for bit the restatement
    (pinned to the reference's CPU scorer by the fixture), slot order and pads included."""
    st = _st()
    words = ivf.pack_mask_high_first(FUSED["mask"])
    kw = {"scaled": dict(per_embedding_scale=FUSED["scale"]),
          "scaled_div": dict(per_embedding_scale=FUSED["scale"], divisor_for_int8=16),
          "index_i32": dict(filtering_bit_mask=words, filtering_bit_index=FUSED["mask_index"]),
          "index_scaled": dict(filtering_bit_mask=words, filtering_bit_index=FUSED["mask_index"],
                               per_embedding_scale=FUSED["scale"], invalid_index_value=-5)}[case]
    dev = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() if isinstance(v, np.ndarray) else v
           for k, v in kw.items()}
    t = [torch.from_numpy(np.ascontiguousarray(FUSED[k])).cuda() for k in ("offsets", "probe", "lengths", "codes", "q")]
    width = int(FUSED["width"])
    raw, idx = st.fused_kmean_ann(*t, width, **dev)
    want_r, want_i = ivf.fused_kmean_ann(FUSED["q"], FUSED["offsets"], FUSED["probe"], FUSED["lengths"],
                                         FUSED["codes"], width, **kw)
    got_r = raw.cpu().numpy()
    assert got_r.dtype == want_r.dtype
    bits = np.uint16 if got_r.dtype == np.float16 else np.int32
    assert np.array_equal(got_r.view(bits), want_r.view(bits)) and np.array_equal(idx.cpu().numpy(), want_i)


@pytest.mark.gpu
def test_fused_kmean_ann_scale_rounds_large_dots_like_the_cuda_scorer():
    """Full-range codes (dots up to ~10^6 at D = 64): the scaled raw is
    fp16(fp32(fp16(dot)) / scale), the CUDA scorer's order, bit for bit; and a partial-mask call
    whose rows read the partial masks of other rows through filtering_bit_index."""
    st = _st()
    rng = np.random.default_rng(31)
    sizes = rng.integers(0, 300, 30)
    offsets = np.r_[0, np.cumsum(sizes)].astype(np.int64)
    n, d, b, p = int(offsets[-1]), 64, 20, 5
    codes = rng.integers(-128, 128, (n, d), dtype=np.int8)
    q = rng.integers(-128, 128, (b, d), dtype=np.int8)
    probe = np.argsort(rng.random((b, 30)), axis=1)[:, :p].astype(np.int64)
    lengths = sizes[probe].astype(np.int64)
    width = int(lengths.sum(1).max())
    scale = (rng.random(n) * 8 + 0.01).astype(np.float16)
    t = [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (offsets, probe, lengths, codes, q)]
    raw, idx = st.fused_kmean_ann(*t, width, per_embedding_scale=torch.from_numpy(scale).cuda())
    want_r, want_i = ivf.fused_kmean_ann(q, offsets, probe, lengths, codes, width, per_embedding_scale=scale)
    assert np.array_equal(raw.cpu().numpy().view(np.uint16), want_r.view(np.uint16))
    assert np.array_equal(idx.cpu().numpy(), want_i)
    # partial masks of 7 "mask rows" (ranges of row r's probes), rows mapped onto them
    mask = rng.random((7, n)) < 0.5
    words = ivf.pack_mask_high_first(mask)
    rows_map = rng.integers(0, 7, b).astype(np.int64)
    sel_rows = np.arange(7) % b
    sel_off, sel_len = offsets[probe[sel_rows]], lengths[sel_rows]
    counts, _, first = ivf.column_info(sel_off, sel_len)
    cumsum = np.cumsum(counts, dtype=np.int32)
    chunks = []
    for i in range(7 * p):
        start, cnt = int(sel_off.reshape(-1)[i]) // 64, int(counts[i])
        chunks.append(words[i // p, start:start + cnt])
    resp = np.concatenate(chunks).astype(np.int64)
    # rows whose mask row holds the same probes as themselves see their own ranges
    probe2 = probe.copy()
    probe2[:] = probe[sel_rows[rows_map]]
    lengths2 = sizes[probe2].astype(np.int64)
    t2 = [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (offsets, probe2, lengths2, codes, q)]
    part = [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (cumsum, first, resp)]
    w2 = int(lengths2.sum(1).max())
    raw2, idx2 = st.fused_kmean_ann_with_partial_masks(*t2, w2, *part,
                                                       filtering_bit_index=torch.from_numpy(rows_map).cuda())
    want2 = ivf.fused_kmean_ann(q, offsets, probe2, lengths2, codes, w2, filtering_bit_mask=words[rows_map])
    assert np.array_equal(raw2.cpu().numpy(), want2[0]) and np.array_equal(idx2.cpu().numpy(), want2[1])


@pytest.mark.gpu
@pytest.mark.parametrize("grouped", [False, True])
def test_search_replays_in_a_cuda_graph(grouped):
    """st::search allocates only through the caller's allocator and never waits on the host, so it
    captures into a CUDA graph (the reference's capture test, test_silvertorch_compile.py:196-270):
    replays with new query values equal eager calls, bit for bit."""
    _st()
    from retrieve_b200 import st

    g, meta = _case(3)
    t = {key: torch.from_numpy(np.ascontiguousarray(g[key])).cuda()
         for key in ("query", "probe", "offsets", "sizes", "codes", "sort_perm")}
    gs = torch.from_numpy(g["gs"]).cuda()
    fn = st.search_grouped if grouped else st.search_rows
    q = t["query"].clone()

    def call():
        return fn(q, t["probe"], t["offsets"], t["sizes"], t["codes"], t["sort_perm"], gs, meta["k"], meta["width"])

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            call()  # warm-up outside the capture
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ids_g, scores_g = call()
    gen = torch.Generator(device="cuda").manual_seed(4)
    for _ in range(3):
        q.copy_(torch.randn(q.shape, generator=gen, device="cuda"))
        graph.replay()
        ids, scores = call()
        torch.cuda.synchronize()
        assert torch.equal(ids_g, ids) and torch.equal(scores_g, scores)
    del graph


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,fmt", [(torch.float32, "fp32"), (torch.float16, "fp16"), (torch.bfloat16, "bf16")])
@pytest.mark.parametrize("d", [64, 96, 192, 256])
def test_fused_kmean_ann_float_embeddings(dtype, fmt, d):
    """Float embeddings: the CUDA scorer's fused multiply-add chains (one block, 256-byte and
    384-byte blocks, fp16 / bf16 in even / odd lanes), bit for bit the restatement's exact-rounding
    emulation, slot order, pads and mask included."""
    from oracle import fdot

    st = _st()
    if fdot.unit(d, fmt) == 0:
        pytest.skip("no chain for this D (the reference has no kernel for it either)")
    rng = np.random.default_rng(d)
    sizes = rng.integers(0, 70, 9)
    offsets = np.r_[0, np.cumsum(sizes)].astype(np.int64)
    n, b, p = int(offsets[-1]), 3, 3
    x = fdot.to_format(rng.standard_normal((n, d)), fmt)
    q = fdot.to_format(rng.standard_normal((b, d)), fmt)
    probe = np.argsort(rng.random((b, 9)), axis=1)[:, :p].astype(np.int64)
    lengths = sizes[probe].astype(np.int64)
    width = int(lengths.sum(1).max())
    mask = rng.random((b, n)) < 0.7
    words = ivf.pack_mask_high_first(mask)
    dev = [torch.from_numpy(np.ascontiguousarray(v)).cuda() for v in (offsets, probe, lengths)]
    xt = torch.from_numpy(x).to(dtype).cuda()
    qt = torch.from_numpy(q).to(dtype).cuda()
    raw, idx = st.fused_kmean_ann(*dev, xt, qt, width, filtering_bit_mask=torch.from_numpy(words).cuda(),
                                  invalid_index_value=-4)
    want_r, want_i = ivf.fused_kmean_ann(q, offsets, probe, lengths, x, width, filtering_bit_mask=words,
                                         invalid_index_value=-4, float_format=fmt)
    assert raw.dtype == dtype
    assert np.array_equal(idx.cpu().numpy(), want_i)
    got = raw.float().cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want_r.astype(np.float32).view(np.uint32))


@pytest.mark.skipif(not REF_CPU_LIB.exists(), reason="the reference's CPU st ops are not built here")
def test_every_reference_st_op_is_served():
    """Every op the reference's SilverTorch build registers under ``st::`` is defined by this
    library alone with the same schema, and gets a CUDA kernel beside the reference's CPU build
    (each in a child process: one registry per process)."""
    import subprocess
    import sys

    listing = (
        "import torch, json\n"
        "{load}\n"
        "ops = sorted(n for n in torch._C._dispatch_get_all_op_names() if n.startswith('st::'))\n"
        "print(json.dumps({{n: str(getattr(torch.ops.st, n[4:].split('.')[0]).default._schema) for n in ops}}))\n"
    )
    root = Path(__file__).resolve().parent.parent

    def run(load):
        r = subprocess.run([sys.executable, "-c", listing.format(load=load)], cwd=root, capture_output=True, text=True,
                           timeout=300)
        assert r.returncode == 0, r.stderr[-2000:]
        import json

        return json.loads(r.stdout.strip().splitlines()[-1])

    ref = run(f"torch.ops.load_library({str(REF_CPU_LIB)!r})")
    ours = run("import retrieve_b200.st")
    assert set(ref) <= set(ours), sorted(set(ref) - set(ours))
    assert all(ours[n] == ref[n] for n in ref)
    code = (
        "import torch\n"
        f"torch.ops.load_library({str(REF_CPU_LIB)!r})\n"
        "import retrieve_b200.st\n"
        "has = torch._C._dispatch_has_kernel_for_dispatch_key\n"
        "missing = [n for n in torch._C._dispatch_get_all_op_names() if n.startswith('st::') and not has(n, 'CUDA')]\n"
        "assert not missing, missing\n"
    )
    r = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]


def _pack_low_first(mask):
    m = np.asarray(mask, dtype=bool)
    b, n = m.shape
    w = (n + 63) // 64
    padded = np.zeros((b, w * 64), dtype=bool)
    padded[:, :n] = m
    return np.bitwise_or.reduce(padded.reshape(b, w, 64).astype(np.uint64) << np.arange(64, dtype=np.uint64),
                                axis=2).view(np.int64)


def _scored_docs(doc, packer, device):
    """The reference's bit-order probe (test_official.py:376-410): one 70-doc cluster (docs 0-63
    in the first mask word and on the warp-aligned path, 64-69 in the second and on the remainder
    path) scored under a mask with exactly ``doc`` set, packed by ``packer``."""
    n, d = 70, 16
    rng = np.random.default_rng(11)
    codes = rng.integers(-128, 128, (n, d), dtype=np.int8)
    q = rng.integers(-128, 128, (1, d), dtype=np.int8)
    mask = np.zeros((1, n), dtype=bool)
    mask[0, doc] = True
    words = packer(mask)
    args = (np.array([0, n]), np.zeros((1, 1), dtype=np.int64), np.array([[n]]))
    if device:
        st = _st()
        t = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (*args, codes, q)]
        _, idx = st.fused_kmean_ann(*t, n, filtering_bit_mask=torch.from_numpy(words).cuda())
        idx = idx.cpu().numpy()
    else:
        _, idx = ivf.fused_kmean_ann(q, args[0], args[1], args[2], codes, n, filtering_bit_mask=words)
    return sorted(idx[idx >= 0].tolist())


@pytest.mark.parametrize("doc", [0, 5, 40, 69])
def test_scorer_reads_the_mask_high_bit_first(doc):
    """The known answer of the reference's T3 test on the restatement: packed high bit first, the
    one set doc and only it is scored; packed low bit first, its mirror in the word (or nothing
    when the mirror lies past the cluster)."""
    assert _scored_docs(doc, ivf.pack_mask_high_first, device=False) == [doc]
    mirror = (doc // 64) * 64 + (63 - doc % 64)
    assert _scored_docs(doc, _pack_low_first, device=False) == ([mirror] if mirror < 70 else [])


@pytest.mark.gpu
@pytest.mark.parametrize("doc", [0, 5, 40, 69])
def test_device_scorer_reads_the_mask_high_bit_first(doc):
    assert _scored_docs(doc, ivf.pack_mask_high_first, device=True) == [doc]
    mirror = (doc // 64) * 64 + (63 - doc % 64)
    assert _scored_docs(doc, _pack_low_first, device=True) == ([mirror] if mirror < 70 else [])
