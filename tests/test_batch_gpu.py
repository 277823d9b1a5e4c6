"""Batched decode of several conversations (cxm_generate_batch) and shared
prefixes held once (cxm_cache_share_prefix), on the GPU.

A batched conversation must get, token for token, what cxm_generate gives it
alone (which the parity tests pin to the oracle), and a cache that borrows a
prefix must behave exactly as one holding a copy. Prompt lengths cover the
three row classes of the reference's matmul dispatch (1-4, 5-23, 24+
tokens), and the formats with a minimum (Q4_K, Q5_K, Q2_K), whose one-row
order differs from the buffered one in the tensor-core epilogue."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _seeded(seed, n, vocab):
    from cosxamix_b200 import serving
    return serving.seeded_tokens(seed, n, vocab)


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    import cosxamix_b200 as cx
    p = str(tmp_path_factory.mktemp("batch") / "tiny.gguf")
    cx.synth_write(p, cx.synth_spec("tiny", seed=42))
    return cx.Modelo(p)


def _single(m, prompt, n_new, prefix=None, plen=0, copy=False):
    import cosxamix_b200 as cx
    c = m.cache(256)
    if prefix is not None:
        (c.copiar_prefijo if copy else c.compartir_prefijo)(prefix, plen)
    return m.generar(prompt, n_new, cx.Muestreador.voraz(), c), c


def test_shared_prefix_equals_copied_prefix(tiny):
    import cosxamix_b200 as cx
    m = tiny
    V = m.cfg.vocab
    lender = m.cache(256)
    m.forward(_seeded(1, 40, V), lender)  # a 40-token prompt: the tensor-core prefill
    suffix = _seeded(2, 9, V)
    toks_copy, c_copy = _single(m, suffix, 20, lender, 40, copy=True)
    toks_share, c_share = _single(m, suffix, 20, lender, 40)
    assert toks_share == toks_copy
    assert len(c_share) == len(c_copy) == 40 + 9 + 20
    for layer in (0, m.cfg.n_layer - 1):
        np.testing.assert_array_equal(c_share.capa(layer), c_copy.capa(layer))
        np.testing.assert_array_equal(c_share.capa(layer, v=True), c_copy.capa(layer, v=True))
    # the lent positions stay as they are while borrowed
    with pytest.raises(ValueError, match="lent"):
        lender.truncar(10)
    with pytest.raises(ValueError, match="lent"):
        lender.limpiar()
    lender.truncar(40)  # at the lent length: nothing moves
    # freed first, the lender lives on for its borrower
    del lender
    import gc
    gc.collect()
    again = m.forward([int(suffix[0])], c_share)
    ref = m.forward([int(suffix[0])], c_copy)
    np.testing.assert_array_equal(again, ref)


def test_prefix_of_a_borrower_comes_from_its_lender(tiny):
    m = tiny
    V = m.cfg.vocab
    lender = m.cache(256)
    m.forward(_seeded(3, 30, V), lender)
    mid = m.cache(256)
    mid.compartir_prefijo(lender, 30)
    m.forward(_seeded(4, 6, V), mid)
    leaf = m.cache(256)
    with pytest.raises(ValueError, match="borrows"):
        leaf.compartir_prefijo(mid, 36)
    leaf.compartir_prefijo(mid, 25)  # within mid's borrowed positions: from the lender
    flat = m.cache(256)
    flat.copiar_prefijo(lender, 25)
    a = m.forward(_seeded(5, 3, V), leaf)
    b = m.forward(_seeded(5, 3, V), flat)
    np.testing.assert_array_equal(a, b)
    # a copy of a borrower reads the lent rows from the lender
    cp = m.cache(256)
    cp.copiar_prefijo(mid, 36)
    np.testing.assert_array_equal(cp.capa(1), mid.capa(1))


@pytest.mark.parametrize("fmt", ["tiny", "q5k", "q2k"])
def test_batch_generate_equals_one_at_a_time(tmp_path_factory, fmt):
    import cosxamix_b200 as cx
    if fmt == "tiny":
        p = str(tmp_path_factory.mktemp("bt") / "t.gguf")
        cx.synth_write(p, cx.synth_spec("tiny", seed=42))
    else:
        t = {"q5k": 13, "q2k": 10}[fmt]
        p = str(tmp_path_factory.mktemp("bt") / f"{fmt}.gguf")
        cx.synth_write(p, cx.synth_spec("tiny", seed=5, type=t, tied=1, n_layer=3))
    m = cx.Modelo(p)
    V = m.cfg.vocab
    lender = m.cache(256)
    m.forward(_seeded(11, 32, V), lender)
    # prompts of 3, 12 and 40 tokens (the three row classes); two conversations borrow the prefix
    specs = [(3, None), (12, None), (40, None), (7, 32), (26, 32)]
    prompts = [_seeded(20 + i, n, V) for i, (n, _) in enumerate(specs)]
    n_new = 24
    want = []
    for pr, (_, pl) in zip(prompts, specs):
        toks, _ = _single(m, pr, n_new, lender if pl else None, pl or 0)
        want.append(toks)
    caches = []
    for _, pl in specs:
        c = m.cache(256)
        if pl:
            c.compartir_prefijo(lender, pl)
        caches.append(c)
    got = m.generar_lote(prompts, n_new, caches)
    assert got == want
    for c, pr, (_, pl) in zip(caches, prompts, specs):
        assert len(c) == (pl or 0) + len(pr) + n_new
    # the caches hold what the single path leaves: one more token continues alike
    c1 = m.cache(256)
    m.generar(prompts[1], n_new, cx.Muestreador.voraz(), c1)
    np.testing.assert_array_equal(m.forward([5], caches[1]), m.forward([5], c1))


def test_batch_against_the_oracle(tiny):
    from oracle import oracle as orc
    m = tiny
    V = m.cfg.vocab
    om = orc.Model(m.ruta)
    prompts = [_seeded(31, 6, V), _seeded(32, 25, V)]
    caches = [m.cache(128), m.cache(128)]
    got = m.generar_lote(prompts, 16, caches)
    for pr, toks in zip(prompts, got):
        want = om.generate(orc.Cache(om), pr, 16, orc.Sampler(0, 0.0, 1.0))
        assert toks == list(want)


def test_batch_stops_each_conversation_at_its_eos(tmp_path_factory):
    import cosxamix_b200 as cx
    base = str(tmp_path_factory.mktemp("eosb") / "b.gguf")
    cx.synth_write(base, cx.synth_spec("tiny", seed=42, n_layer=2))
    mb = cx.Modelo(base)
    V = mb.cfg.vocab
    prompts = [_seeded(41, 5, V), _seeded(42, 8, V), _seeded(43, 30, V)]
    free = mb.generar_lote(prompts, 20, [mb.cache(128) for _ in prompts])
    eos = free[1][6]  # the second conversation's 7th token becomes the eos
    p = str(tmp_path_factory.mktemp("eosb") / "e.gguf")
    cx.synth_write(p, cx.synth_spec("tiny", seed=42, n_layer=2, eos=eos))
    m = cx.Modelo(p)
    caches = [m.cache(128) for _ in prompts]
    got = m.generar_lote(prompts, 20, caches)
    for z, pr in enumerate(prompts):
        want, c = _single(m, pr, 20)
        assert got[z] == want
        assert len(caches[z]) == len(c)
    assert got[1] == free[1][:6]


def test_batch_qwen3b_shared_prefix(tmp_path_factory):
    """The headline shape: a 512-token shared prefix, 3 conversations with
    64-token suffixes, 16 greedy tokens each, batched == one at a time."""
    import bench
    import cosxamix_b200 as cx
    m = cx.Modelo(bench.ensure_model("qwen3b", 42))
    V = m.cfg.vocab
    lender = m.cache(640)
    m.forward(bench.seeded_prompt(42, 512, V), lender)
    prompts = [_seeded(60 + z, 64, V) for z in range(3)]
    want = []
    for pr in prompts:
        c = m.cache(640)
        c.compartir_prefijo(lender, 512)
        want.append(m.generar(pr, 16, cx.Muestreador.voraz(), c))
    caches = []
    for _ in prompts:
        c = m.cache(640)
        c.compartir_prefijo(lender, 512)
        caches.append(c)
    assert m.generar_lote(prompts, 16, caches) == want
