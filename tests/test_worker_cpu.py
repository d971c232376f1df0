"""The drop-in boundary on CPU: plugin registration (tri_sds/__init__.py:1-10)
and TriSDSWorker's dispatch (tri_sds/worker.py:9-68) with a stand-in engine
that records its calls (no GPU, no kernels)."""
import pytest
import torch


class FakeEngine:
    """The engine interface the worker drives: prepare / step / run_draft /
    run_verify, with a tokens buffer of shape [B, depth+2]."""

    def __init__(self, B=2, width=7):
        self.calls = []
        self.tokens = torch.full((B, width), -1, dtype=torch.int64)
        self.accept_len = torch.zeros(B, dtype=torch.int32)

    def prepare(self, prompt, lengths=None):
        self.calls.append(("prepare", tuple(prompt.shape)))
        self.prompt, self.lengths = prompt, lengths
        return prompt[:, -1]

    def step(self, U=None):
        self.calls.append(("step",))
        self.tokens[:, 0] = len(self.calls)
        return self.tokens, self.accept_len

    def step_host(self, cur_host, tokens_host, accept_host):
        self.calls.append(("step_host",))
        tokens_host.copy_(self.tokens)
        accept_host.copy_(self.accept_len)
        return tokens_host, accept_host

    def run_draft(self):
        self.calls.append(("draft",))
        return torch.arange(8).reshape(2, 4)

    def run_verify(self):
        self.calls.append(("verify",))
        return self.tokens, self.accept_len


def test_create_plugin_registers_the_replacement():
    import tri_sds_b200
    from tri_sds_b200.sglang_compat import HAVE_SGLANG, HookRegistry, HookType
    from tri_sds_b200.worker import TriSDSWorker
    if HAVE_SGLANG:
        pytest.skip("SGLang's own registry is installed")
    tri_sds_b200.create_plugin()
    assert HookRegistry.lookup(tri_sds_b200.STANDALONE_WORKER) == (TriSDSWorker, HookType.REPLACE)
    assert tri_sds_b200.STANDALONE_WORKER == "sglang.srt.speculative.standalone_worker.StandaloneWorker"


def test_sds_disabled_delegates_to_sglang(monkeypatch):
    from tri_sds_b200.sglang_compat import HAVE_SGLANG, ScheduleBatch
    from tri_sds_b200.worker import TriSDSWorker
    if HAVE_SGLANG:
        pytest.skip("needs the stand-in base class")
    monkeypatch.delenv("SDS_ENABLED", raising=False)
    w = TriSDSWorker()
    eng = FakeEngine()
    w.attach_engine(eng)
    batch = ScheduleBatch(input_ids=torch.zeros(2, 5, dtype=torch.int64))
    for meth in (w.forward_batch_generation, w.draft, w.verify):
        with pytest.raises(NotImplementedError):
            meth(batch)
    assert eng.calls == []


def test_sds_enabled_runs_the_engine(monkeypatch):
    from tri_sds_b200.sglang_compat import ScheduleBatch
    from tri_sds_b200.worker import TriSDSWorker
    monkeypatch.setenv("SDS_ENABLED", "1")
    w = TriSDSWorker()
    eng = FakeEngine()
    w.attach_engine(eng)
    prompt = torch.randint(0, 100, (2, 5))
    toks, n = w.forward_batch_generation(ScheduleBatch(input_ids=prompt))
    # the first call prefills from the prompt, then runs one cycle
    assert eng.calls == [("prepare", (2, 5)), ("step",)]
    assert toks.shape == (2, 7) and n.shape == (2,)
    # results are copies: the next cycle does not overwrite them
    first = toks.clone()
    w.forward_batch_generation(ScheduleBatch(input_ids=prompt))
    assert eng.calls[-1] == ("step",) and eng.calls.count(("prepare", (2, 5))) == 1
    assert torch.equal(toks, first)
    assert w.draft(ScheduleBatch(input_ids=prompt)).shape == (2, 4)
    w.verify(ScheduleBatch(input_ids=prompt))
    assert eng.calls[-2:] == [("draft",), ("verify",)]


def test_worker_without_engine_says_so(monkeypatch):
    from tri_sds_b200.sglang_compat import ScheduleBatch
    from tri_sds_b200.worker import TriSDSWorker
    monkeypatch.setenv("SDS_ENABLED", "1")
    with pytest.raises(RuntimeError, match="attach_engine"):
        TriSDSWorker().forward_batch_generation(ScheduleBatch(input_ids=torch.zeros(1, 3, dtype=torch.int64)))


def test_status_watch_raises_on_a_device_error():
    """The engines read their kernels' status words with every host-driven
    cycle: a nonzero word (a bounded device wait that gave up) raises and is
    cleared."""
    from tri_sds_b200.model import StatusWatch
    words = [torch.zeros(1, dtype=torch.int32), torch.tensor([5], dtype=torch.int32)]
    w = StatusWatch(words)
    w.copy()
    with pytest.raises(RuntimeError, match="status 5"):
        w.check()
    assert int(words[1]) == 0
    w.copy()
    w.check()   # clean now


def test_ragged_prompts_reach_the_engine_padded_with_their_lengths(monkeypatch):
    """SGLang batches hold prompts of different lengths: a list of prompts is
    padded behind each prompt and the lengths go with it; a padded [B, P]
    tensor carries them in seq_lens; full rows need none."""
    from tri_sds_b200.sglang_compat import ScheduleBatch
    from tri_sds_b200.worker import TriSDSWorker, prompt_tensor
    monkeypatch.setenv("SDS_ENABLED", "1")
    w = TriSDSWorker()
    eng = FakeEngine(B=3)
    w.attach_engine(eng)
    w.forward_batch_generation(ScheduleBatch(input_ids=[[5, 6, 7], [8], [9, 10, 11, 12]]))
    assert eng.calls[0] == ("prepare", (3, 4))
    assert eng.prompt.tolist() == [[5, 6, 7, 0], [8, 0, 0, 0], [9, 10, 11, 12]]
    assert eng.lengths.tolist() == [3, 1, 4]
    ids, n = prompt_tensor(ScheduleBatch(input_ids=torch.ones(2, 6, dtype=torch.int64), seq_lens=[6, 2]))
    assert ids.shape == (2, 6) and n.dtype == torch.int32 and n.tolist() == [6, 2]
    ids, n = prompt_tensor(ScheduleBatch(input_ids=[[1, 2], [3, 4]]))
    assert ids.tolist() == [[1, 2], [3, 4]] and n is None
    ids, n = prompt_tensor(ScheduleBatch(input_ids=[1, 2, 3]))
    assert ids.shape == (1, 3) and n is None
    with pytest.raises(ValueError):
        prompt_tensor(ScheduleBatch(input_ids=[[1], []]))


def test_worker_follows_the_batch_it_is_given(monkeypatch):
    """A later batch with new prompts (or other request ids) prefills the
    engine again; the same prompt or one current token per sequence
    continues; a batch of another size is refused before anything runs."""
    from types import SimpleNamespace

    from tri_sds_b200.sglang_compat import ScheduleBatch
    from tri_sds_b200.worker import TriSDSWorker
    monkeypatch.setenv("SDS_ENABLED", "1")
    w = TriSDSWorker()
    eng = FakeEngine()
    w.attach_engine(eng)
    p1 = torch.randint(0, 100, (2, 5), generator=torch.Generator().manual_seed(1))
    p2 = torch.randint(0, 100, (2, 6), generator=torch.Generator().manual_seed(2))
    w.forward_batch_generation(ScheduleBatch(input_ids=p1))
    w.forward_batch_generation(ScheduleBatch(input_ids=p1))
    w.forward_batch_generation(ScheduleBatch(input_ids=torch.tensor([[3], [4]])))
    assert [c for c in eng.calls if c[0] == "prepare"] == [("prepare", (2, 5))]
    # new prompts: prepared again from them
    w.forward_batch_generation(ScheduleBatch(input_ids=p2))
    assert eng.calls[-2:] == [("prepare", (2, 6)), ("step",)]
    assert torch.equal(eng.prompt, p2)
    # the same prompt shape with other ids is a new batch too
    p3 = p2.clone()
    p3[0, 0] += 1
    w.forward_batch_generation(ScheduleBatch(input_ids=p3))
    assert eng.calls[-2] == ("prepare", (2, 6)) and torch.equal(eng.prompt, p3)
    # request identities decide when the batch carries them
    reqs = [SimpleNamespace(rid="a"), SimpleNamespace(rid="b")]
    w.forward_batch_generation(ScheduleBatch(input_ids=p1, reqs=reqs))
    n_prep = sum(c[0] == "prepare" for c in eng.calls)
    w.forward_batch_generation(ScheduleBatch(input_ids=torch.tensor([[3], [4]]), reqs=list(reqs)))
    assert sum(c[0] == "prepare" for c in eng.calls) == n_prep
    w.forward_batch_generation(ScheduleBatch(input_ids=p1, reqs=[SimpleNamespace(rid="c"), reqs[1]]))
    assert sum(c[0] == "prepare" for c in eng.calls) == n_prep + 1
    # another batch size: refused, the engine untouched
    before = list(eng.calls)
    with pytest.raises(ValueError, match="engine serves 2"):
        w.forward_batch_generation(ScheduleBatch(input_ids=torch.zeros(3, 4, dtype=torch.int64)))
    assert eng.calls == before


def test_status_error_clears_the_counters_and_retires_a_peer_group():
    """After a device wait gave up, the word and the tile counters beside it
    (the workspace header) are zeroed so the next launch starts afresh, and a
    peer group is retired: its ranks' per-CTA epochs no longer agree."""
    from tri_sds_b200.model import StatusWatch
    ws = torch.arange(64, dtype=torch.uint8)           # header = first 32 bytes
    ws[:4] = torch.tensor([5, 0, 0, 0], dtype=torch.uint8)
    retired = []
    w = StatusWatch([(ws[:4].view(torch.int32), ws[:32], lambda: retired.append(1))])
    w.copy()
    with pytest.raises(RuntimeError, match="status 5"):
        w.check()
    assert retired == [1]
    assert int(ws[:32].sum()) == 0 and torch.equal(ws[32:], torch.arange(32, 64, dtype=torch.uint8))
    w.copy()
    w.check()


def test_retired_peer_group_refuses_the_next_cycle():
    from types import SimpleNamespace

    from tri_sds_b200.model import QwenModel
    m = QwenModel.__new__(QwenModel)
    m.peer = SimpleNamespace(broken=False)
    m.ensure_usable()
    m._retire_peer()
    with pytest.raises(RuntimeError, match="retired"):
        m.ensure_usable()
