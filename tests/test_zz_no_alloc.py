"""ge_pool_head_noalloc against the forward's own pooling and head.

Some callers cannot allocate device memory (a plugin whose host runtime owns every device
allocation, or a serving loop that must not trigger an allocation mid-request), so the library
offers the forward's last stage -- mean-pool, then the dense head -- over caller-owned device
buffers with its intermediates in a static device array.  This test feeds it the final-normed
hidden states of two batches, one call after the other, and checks each output against the
pooled vectors that ge_forward_packed (which uses its allocated workspace) returns for the same
sequences.  This file is named to run after every other test file.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-4  # max |got - want| / max |want|, the kernel tolerance of the other GPU tests


@pytest.fixture(scope="module", params=["gemma-embedding", "gemma-embedding2"])
def model(request, ge, synth, cuda_device):
    """gemma-embedding takes the dense-head branch (768 -> 3072 -> 768), gemma-embedding2 the
    per-token output projection (512 -> 768)."""
    path = synth.model_path(request.param, seed=1, layers=6, vocab=4096)
    m = ge.EmbeddingModel.load(path)
    yield m
    m.close()


def run_noalloc(model, seqs, pairs=None, ntok=None):
    import torch

    hidden = np.concatenate([model.trace(s, -1) for s in seqs])  # result_norm rows of each sequence
    lens = [len(s) for s in seqs]
    if pairs is None:
        starts = np.concatenate([[0], np.cumsum(lens)[:-1]])
        pairs = np.stack([starts, lens], axis=1).astype(np.int32)
    d_hidden = torch.from_numpy(hidden).cuda()
    d_seqs = torch.from_numpy(np.asarray(pairs, np.int32)).cuda()
    d_out = torch.full((len(pairs), model.info.output_dimensions), float("nan"), device="cuda")
    torch.cuda.synchronize()
    model.pool_head_noalloc(d_hidden, hidden.shape[0] if ntok is None else ntok, d_seqs, len(pairs), d_out)
    torch.cuda.synchronize()
    return d_out.cpu().numpy(), hidden


def test_noalloc_head_matches_forward_on_two_calls(model, synth, ge):
    first = synth.random_sequences([5, 130, 257, 64], seed=31, vocab=4096)
    second = synth.random_sequences([300, 17, 41], seed=32, vocab=4096)
    for seqs in (first, second):
        want = model.embed_tokens(seqs)
        got, _ = run_noalloc(model, seqs)
        assert not np.isnan(got).any()
        rel = float(np.abs(got - want).max() / np.abs(want).max())
        assert rel < TOL, rel


def test_noalloc_reads_only_rows_below_ntok(model, synth):
    """Ranges come from the caller's device memory: one that runs past ntok is cut there, and
    one with no row inside pools to zeros, so the head returns its value at zero -- and no
    memory past the caller's rows is read."""
    seqs = synth.random_sequences([40, 90], seed=33, vocab=4096)
    exact, _ = run_noalloc(model, seqs, pairs=[[0, 40], [40, 50]], ntok=90)
    zero, _ = run_noalloc(model, seqs, pairs=[[0, 0], [0, 0]])
    # (40, 10_000) is cut at ntok = 90, so it pools the same rows as (40, 50); (90, 5) and
    # (0, 0) hold no row.
    got, _ = run_noalloc(model, seqs, pairs=[[0, 40], [40, 10_000], [90, 5], [0, 0]], ntok=90)
    assert not np.isnan(got).any()
    assert np.array_equal(got[:2], exact)
    want = model.embed_tokens(seqs[:1])[0]
    assert float(np.abs(got[0] - want).max() / np.abs(want).max()) < TOL
    assert np.array_equal(got[2], zero[0]) and np.array_equal(got[3], zero[0])


def test_noalloc_rejects_more_sequences_than_its_scratch_holds(model, ge):
    import torch

    n = 129
    d_hidden = torch.zeros((n, model.info.hidden_size), device="cuda")
    d_seqs = torch.tensor([[i, 1] for i in range(n)], dtype=torch.int32, device="cuda")
    d_out = torch.zeros((n, model.info.output_dimensions), device="cuda")
    with pytest.raises(ge.GemmaEmbedError) as e:
        model.pool_head_noalloc(d_hidden, n, d_seqs, n, d_out)
    assert e.value.case == "invalidOptions"
    assert "128" in e.value.message
