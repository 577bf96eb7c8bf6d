"""Full-forward parity on the GPU: ``CudaBackend.forward`` (through the C ABI) against the CPU
oracle of the reference forward on identical seeded weights and token ids.

Tolerances (stated by the task for this path, tighter than the reference's own
``laya-mlx/tests/parity.rs:29-39`` logits < 0.15 / probs < 0.02):
  * per-question probabilities within 1e-2 absolute,
  * final encoder hidden states within 2e-2 relative (Frobenius, over the real tokens),
  * choice argmax equal wherever the fp32 top-two margin exceeds the measured logit error,
  * masked marker slots exactly -1e4.
"""
import numpy as np
import pytest

from sys1rust_b200.batch import Batch, EncodedItem, Varlen, collate_to

pytestmark = pytest.mark.gpu

HIDDEN_REL = 2e-2
PROB_ABS = 1e-2


def make_rows(cfg, seed, lens, ks, qtypes=None):
    rng = np.random.Generator(np.random.PCG64(seed))
    items = []
    for i, (L, k) in enumerate(zip(lens, ks)):
        ids = rng.integers(4, cfg.encoder.vocab_size, size=L).astype(np.uint32)
        ids[0] = 1
        if L > 1:
            ids[-1] = 2
        k = min(k, max(L - 1, 0))
        markers = sorted(rng.choice(np.arange(1, L), size=k, replace=False).tolist()) if k else []
        qt = int(qtypes[i]) if qtypes is not None else int(rng.integers(0, 3))
        items.append(EncodedItem(ids.tolist(), markers, qt))
    return items


def oracle(cfg, w, batch, emulate=False):
    from oracle.forward_ref import OracleModel
    return OracleModel(cfg, w.tensors, emulate_bf16=emulate).forward(batch)


def question_probs(logits, batch):
    out = []
    for r in range(batch.n):
        c = int(batch.marker_count[r])
        if c:
            z = logits[r * batch.kmax: r * batch.kmax + c].astype(np.float64)
            z = np.exp(z - z.max())
            out.append(z / z.sum())
    return out


def check_against_oracle(cfg, w, be, batch):
    got = be.forward(batch)
    hid = be.encoder_hidden(batch).reshape(batch.n, batch.len, -1)
    lo, po, ho = oracle(cfg, w, batch)
    am = batch.attention_mask.reshape(batch.n, batch.len).astype(bool)
    # hidden state
    rel = np.linalg.norm(hid[am] - ho[am]) / np.linalg.norm(ho[am])
    assert rel < HIDDEN_REL, f"hidden rel err {rel}"
    # masked slots
    for r in range(batch.n):
        for k in range(int(batch.marker_count[r]), batch.kmax):
            assert got.logits[r * batch.kmax + k] == np.float32(-1e4)
    # probabilities per question
    for pg, pw in zip(question_probs(got.logits, batch), question_probs(lo, batch)):
        assert np.abs(pg - pw).max() < PROB_ABS
    # argmax: equal to the oracle's wherever its top-two margin exceeds twice the measured logit
    # error; in every row the option picked has an oracle logit within that error of the best
    err = float(np.abs(got.logits - lo).max()) if got.logits.size else 0.0
    for r in range(batch.n):
        c = int(batch.marker_count[r])
        if c >= 2:
            z = lo[r * batch.kmax: r * batch.kmax + c]
            gi = int(np.argmax(got.logits[r * batch.kmax: r * batch.kmax + c]))
            assert z[gi] >= z.max() - 2 * err
            srt = np.sort(z)
            if srt[-1] - srt[-2] > 2 * err:
                assert gi == np.argmax(z)
    assert np.all(np.isfinite(got.pooled))
    prel = np.linalg.norm(got.pooled - po) / np.linalg.norm(po)
    assert prel < 5e-2, f"pooled rel err {prel}"
    return rel, err


def test_small_model_matches_oracle(cuda_lib):
    from conftest import get_backend
    cfg, w, be = get_backend("small:3")
    items = make_rows(cfg, 21, [1, 2, 9, 17, 40, 64, 65, 130, 300], [0, 1, 2, 3, 4, 2, 5, 3, 6])
    batch = collate_to(items, cfg.encoder.pad_token_id)
    check_against_oracle(cfg, w, be, batch)


def test_large_model_matches_oracle(cuda_lib):
    from conftest import get_backend
    cfg, w, be = get_backend("large:0")
    items = make_rows(cfg, 22, [128, 37, 200, 300], [2, 3, 4, 9], qtypes=[2, 0, 1, 0])
    batch = collate_to(items, cfg.encoder.pad_token_id)
    rel, err = check_against_oracle(cfg, w, be, batch)
    print(f"large: hidden rel {rel:.4g}, logit max err {err:.4g}")


def test_large_model_long_rows(cuda_lib):
    """Rows at 511/512/513 tokens and one long row (window and global paths over many tiles)."""
    from conftest import get_backend
    cfg, w, be = get_backend("large:0")
    items = make_rows(cfg, 23, [511, 512, 513, 1024], [3, 1, 2, 10])
    batch = collate_to(items, cfg.encoder.pad_token_id)
    check_against_oracle(cfg, w, be, batch)


@pytest.mark.parametrize("model,mode", [("small:3", "tc"), ("small:3", "mma"), ("large:0", "tc")])
def test_attention_settings_match_oracle(cuda_lib, model, mode):
    """The forward with each attention setting forced everywhere (the default `attn=auto` runs the
    tcgen05 kernel on full rows when its grid fills the SMs, else and on the pruned head rows the
    mma.sync kernel)."""
    import os
    from sys1rust_b200.backend import CudaBackend
    from conftest import get_backend
    cfg, w, _ = get_backend(model)
    old = os.environ.get("S1C_SETTINGS")
    os.environ["S1C_SETTINGS"] = (old + "," if old else "") + f"attn={mode}"
    try:
        be = CudaBackend.from_synthetic(cfg, w.tensors)
    finally:
        if old is None:
            del os.environ["S1C_SETTINGS"]
        else:
            os.environ["S1C_SETTINGS"] = old
    try:
        items = make_rows(cfg, 24, [1, 2, 9, 17, 40, 64, 65, 130, 300, 700], [0, 1, 2, 3, 4, 2, 5, 3, 6, 9])
        check_against_oracle(cfg, w, be, collate_to(items, cfg.encoder.pad_token_id))
    finally:
        be.close()


def test_rows_agree_alone_or_batched(cuda_lib):
    """A row's outputs alone and inside a batch (``laya-core/src/agent.rs:400-442`` checks
    batch-vs-single agreement). Alone, a short row runs its GEMMs split over K, so the fp32 sums
    are grouped differently: the outputs agree to rounding, not bit for bit."""
    from conftest import get_backend
    cfg, w, be = get_backend("large:0")
    items = make_rows(cfg, 24, [50, 129, 7, 260], [2, 3, 1, 4])
    batch = collate_to(items, cfg.encoder.pad_token_id)
    full = be.forward(batch)
    d = cfg.encoder.hidden_size
    for r, it in enumerate(items):
        one = collate_to([it], cfg.encoder.pad_token_id, min_len=0)
        o = be.forward(one)
        k = len(it.markers)
        assert np.abs(o.logits[:k] - full.logits[r * batch.kmax: r * batch.kmax + k]).max() < 2e-3
        ref = full.pooled[r * d:(r + 1) * d]
        assert np.linalg.norm(o.pooled - ref) / np.linalg.norm(ref) < 1e-2


def test_forward_is_reproducible(cuda_lib):
    """The same batch gives the same outputs bit for bit, run after run (split-K partial sums are
    added in a fixed order)."""
    from conftest import get_backend
    cfg, w, be = get_backend("large:0")
    for lens in ([50], [129, 7, 260]):
        batch = collate_to(make_rows(cfg, 28, lens, [2] * len(lens)), cfg.encoder.pad_token_id)
        outs = [be.forward(batch) for _ in range(4)]
        for o in outs[1:]:
            assert np.array_equal(o.logits, outs[0].logits) and np.array_equal(o.pooled, outs[0].pooled)


def test_padded_and_varlen_entry_points_agree(cuda_lib):
    from conftest import get_backend
    cfg, w, be = get_backend("small:3")
    items = make_rows(cfg, 25, [5, 33, 12], [2, 0, 3])
    batch = collate_to(items, cfg.encoder.pad_token_id)
    a = be.forward(batch)
    b = be.forward_varlen(Varlen.from_batch(batch), hidden=True)
    assert np.array_equal(a.logits, b.logits) and np.array_equal(a.pooled, b.pooled)
    hid = be.encoder_hidden(batch).reshape(batch.n, batch.len, -1)
    am = batch.attention_mask.reshape(batch.n, batch.len).astype(bool)
    # the hook also runs the padding positions near the real tokens, so its GEMMs see more rows:
    # equal to rounding, not bit for bit
    ref = b.hidden.reshape(-1, cfg.encoder.hidden_size)
    assert np.linalg.norm(hid[am] - ref) / np.linalg.norm(ref) < 1e-2


@pytest.mark.parametrize("name", ["small:3", "large:0"])
def test_encoder_hidden_at_padding_positions(cuda_lib, name):
    """``encoder_hidden`` in the padded layout (``lib.rs:1865-1878``): padding positions within the
    sliding window of a real token hold the reference's computed state (the oracle runs the padded
    layout with the -1e4 key mask); positions farther away see only masked keys in the reference's
    window layers and are 0 here."""
    from conftest import get_backend
    cfg, w, be = get_backend(name)
    batch = collate_to(make_rows(cfg, 70, [1, 63, 300], [0, 3, 5]), cfg.encoder.pad_token_id)
    hid = be.encoder_hidden(batch).reshape(batch.n, batch.len, -1)
    _, _, ho = oracle(cfg, w, batch)
    ho = np.asarray(ho).reshape(batch.n, batch.len, -1)
    win = cfg.encoder.window()
    for r, sl in enumerate(batch.seq_lens):
        keep = min(batch.len, int(sl) + win)
        got, want = hid[r, :keep], ho[r, :keep]
        rel = np.linalg.norm(got - want) / np.linalg.norm(want)
        assert rel < HIDDEN_REL, (r, rel)
        pad = slice(int(sl), keep)
        if keep > sl:  # the padding positions alone
            rel_p = np.linalg.norm(hid[r, pad] - ho[r, pad]) / np.linalg.norm(ho[r, pad])
            assert rel_p < HIDDEN_REL, (r, rel_p)
        assert np.all(hid[r, keep:] == 0)


def test_batch_without_markers(cuda_lib):
    from conftest import get_backend
    cfg, w, be = get_backend("small:3")
    batch = collate_to(make_rows(cfg, 26, [10, 3], [0, 0]), cfg.encoder.pad_token_id)
    assert batch.kmax == 0
    out = be.forward(batch)
    assert out.logits.size == 0 and out.pooled.size == 2 * cfg.encoder.hidden_size
    _, po, _ = oracle(cfg, w, batch)
    assert np.linalg.norm(out.pooled - po) / np.linalg.norm(po) < 5e-2
    # an empty batch is a no-op on both entry points
    empty = collate_to([], cfg.encoder.pad_token_id)
    assert empty.n == 0
    out = be.forward(empty)
    assert out.logits.size == 0 and out.pooled.size == 0
    out = be.forward_varlen(Varlen.from_rows([]))
    assert out.logits.size == 0 and out.pooled.size == 0


def test_malformed_batches_are_errors(cuda_lib):
    from conftest import get_backend
    from sys1rust_b200.backend import BackendError
    cfg, w, be = get_backend("small:3")
    good = collate_to(make_rows(cfg, 27, [6, 4], [2, 1]), cfg.encoder.pad_token_id)
    bad_mask = Batch(**{**good.__dict__, "attention_mask": good.attention_mask.copy()})
    bad_mask.attention_mask[good.len - 1] = 0  # row 0 is full length: mask no longer matches
    with pytest.raises(BackendError, match="attention mask"):
        be.forward(bad_mask)
    bad_id = Batch(**{**good.__dict__, "input_ids": good.input_ids.copy()})
    bad_id.input_ids[1] = cfg.encoder.vocab_size + 5
    with pytest.raises(BackendError, match="vocabulary"):
        be.forward(bad_id)
    bad_marker = Batch(**{**good.__dict__, "marker_pos": good.marker_pos.copy()})
    bad_marker.marker_pos[good.kmax] = 10  # row 1 has 4 tokens
    with pytest.raises(BackendError, match="marker"):
        be.forward(bad_marker)
    # a null token array on the host-buffer entry point is an argument error, not a crash
    import ctypes as C
    from sys1rust_b200.backend import S1C_ERR_ARG, lib
    v = Varlen.from_rows(make_rows(cfg, 28, [5], [1]))
    cv, keep = be._cvarlen(v)
    cv.ids = None
    lg = np.zeros(max(v.n * v.kmax, 1), np.float32)
    pl = np.zeros(v.n * cfg.encoder.hidden_size, np.float32)
    rc = lib().s1c_forward_varlen(be._h, C.byref(cv), lg.ctypes.data, pl.ctypes.data, None)
    assert rc == S1C_ERR_ARG and "null" in be._err()
    # the handle stays usable after an error
    out = be.forward(good)
    assert np.all(np.isfinite(out.pooled))


def test_graph_replay_matches_direct_launches(cuda_lib):
    """A shape's third forward replays a captured CUDA graph; its outputs equal, bit for bit, those
    of a backend that launches kernel by kernel (`graphs=0`), also for new data of the same shape."""
    import os
    from sys1rust_b200.backend import CudaBackend
    from conftest import get_backend
    cfg, w, be = get_backend("small:3")
    old = os.environ.get("S1C_SETTINGS")
    os.environ["S1C_SETTINGS"] = (old + "," if old else "") + "graphs=0"
    try:
        direct = CudaBackend.from_synthetic(cfg, w.tensors)
    finally:
        if old is None:
            del os.environ["S1C_SETTINGS"]
        else:
            os.environ["S1C_SETTINGS"] = old
    a = collate_to(make_rows(cfg, 31, [40, 17, 90], [3, 2, 4]), cfg.encoder.pad_token_id)
    b = collate_to(make_rows(cfg, 32, [40, 17, 90], [3, 2, 4]), cfg.encoder.pad_token_id)
    outs = [be.forward(a) for _ in range(3)]  # direct, capture, replay
    ref = direct.forward(a)
    for o in outs:
        assert np.array_equal(o.logits, ref.logits) and np.array_equal(o.pooled, ref.pooled)
    ob, rb = be.forward(b), direct.forward(b)  # replay with new ids and markers
    assert np.array_equal(ob.logits, rb.logits) and np.array_equal(ob.pooled, rb.pooled)
    assert not np.array_equal(ob.pooled, outs[0].pooled)
    direct.close()


def test_tied_options_pick_the_first(cuda_lib):
    """Two marker slots on the same token get bit-identical logits (the same hidden row through the
    same scorer), so their tie is exact on both sides; the answer's argmax is then the first of the
    tied options, as the reference's decode takes the first maximum."""
    from conftest import get_backend
    from sys1rust_b200.batch import EncodedItem
    from sys1rust_b200.decode import ActHead, Temperatures, decode
    cfg, w, be = get_backend("small:3")
    rows = make_rows(cfg, 71, [40, 90], [0, 0])
    best = []
    for it in rows:
        # find the row's best marker position, then offer it twice after a worse option
        probe = EncodedItem(it.ids, list(range(1, len(it.ids) - 1)), 0)
        lg = be.forward(collate_to([probe], cfg.encoder.pad_token_id)).logits
        p_best, p_worse = 1 + int(np.argmax(lg)), 1 + int(np.argmin(lg))
        best.append(EncodedItem(it.ids, [p_worse, p_best, p_best], 0))
    batch = collate_to(best, cfg.encoder.pad_token_id)
    out = be.forward(batch)
    lo, _, _ = oracle(cfg, w, batch)
    for r in range(batch.n):
        z = out.logits[r * batch.kmax: r * batch.kmax + 3]
        assert z[1] == z[2] and z[1] > z[0]
        assert lo[r * batch.kmax + 1] == lo[r * batch.kmax + 2]
        assert int(np.argmax(z)) == 1 == int(np.argmax(lo[r * batch.kmax: r * batch.kmax + 3]))
    d = cfg.encoder.hidden_size
    head = ActHead(np.zeros((4, d + 4), np.float32), np.zeros(4, np.float32), np.zeros((2, 4), np.float32),
                   np.zeros(2, np.float32))
    answers, _ = decode(out.logits, out.pooled, batch.marker_count, batch.qtype, batch.kmax, d, Temperatures(), head)
    assert [a["argmax"] for a in answers] == [1, 1]
