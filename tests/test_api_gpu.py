"""The reference-shaped public API (DFlashGenerator, dflash_generate_stream, adapter
contract) on the GPU, mirroring the reference's own tests/test_streaming.py."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need(lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.fixture(scope="module")
def gen():
    from dflash_b200 import DFlashGenerator
    return DFlashGenerator("random:tiny", "random:tiny")


def test_generate_from_tokens_is_lossless(gen):
    prompt = list(range(5, 69))
    res = gen.generate_from_tokens(prompt, max_new_tokens=40)
    plain = gen.generate_from_tokens(prompt, max_new_tokens=40, speculative_tokens=1)
    assert res.output_tokens == plain.output_tokens
    assert len(res.generated_tokens) == 40
    m = res.metrics
    for key in ("num_input_tokens", "num_output_tokens", "prefill_time_s", "decode_time_s", "total_time_s",
                "prompt_tps", "generation_tps", "end_to_end_tps", "avg_acceptance_length", "acceptance_lengths",
                "peak_memory_gb", "target_cache_summary", "speculative_tokens"):
        assert key in m, key
    assert sum(m["acceptance_lengths"]) >= 39


def test_stream_deltas_reassemble(gen):
    prompt = list(range(7, 40))
    events = list(gen.stream_from_tokens(prompt, max_new_tokens=25))
    assert events[-1].finished and events[-1].metrics is not None
    text = "".join(e.delta for e in events)
    assert text == events[-1].text
    toks = [t for e in events for t in e.token_ids]
    assert toks == events[-1].generated_tokens


def test_stop_token_truncates(gen):
    prompt = list(range(9, 50))
    ref = gen.generate_from_tokens(prompt, max_new_tokens=30)
    stop = ref.generated_tokens[10]
    first = ref.generated_tokens.index(stop)
    gen.target.tokenizer.eos_token_ids = [stop]
    try:
        res = gen.generate_from_tokens(prompt, max_new_tokens=30)
    finally:
        gen.target.tokenizer.eos_token_ids = []
    assert res.generated_tokens == ref.generated_tokens[:first + 1]


def test_adapter_contract_verify_and_rewind(gen):
    """forward_with_hidden_states / lm_head_argmax / rewind_kv_caches behave like the
    reference adapter: a rewound cache recomputes identically."""
    t = gen.target
    cache = t.make_cache(512)
    prompt = torch.tensor(list(range(3, 35)), dtype=torch.int32)[None]
    logits, hid = t.forward_with_hidden_states(prompt, cache, gen.draft.target_layer_ids)
    assert hid.shape == (1, 32, len(gen.draft.target_layer_ids) * t.model.cfg.hidden_size)
    block = torch.tensor([[11, 12, 13, 14]], dtype=torch.int32)
    l1, h1, rec = t.forward_with_hidden_states(block, cache, gen.draft.target_layer_ids, True)
    assert rec == {}
    assert cache.offset == 36
    t.rewind_kv_caches(cache, 3)
    assert cache.offset == 33
    l2, h2 = t.forward_with_hidden_states(block[:, 1:], cache, gen.draft.target_layer_ids)
    assert torch.equal(l2[0], l1[0, 1:])
    assert torch.equal(h2[0], h1[0, 1:])
    am = t.lm_head_argmax(h1.new_zeros(1, 1, t.model.cfg.hidden_size) + 0.1)
    assert am.shape == (1, 1)


def test_batched_stream_matches_single_requests(gen):
    """dflash_generate_batch_stream with three prompts (different lengths and limits) gives
    each prompt's single-request tokens, acceptance record and finish reason."""
    from dflash_b200.runtime import dflash_generate_batch_stream
    prompts = [list(range(5, 69)), list(range(11, 30)), list(range(3, 100, 2))]
    limits = [40, 17, 25]
    singles = [gen.generate_from_tokens(p, max_new_tokens=n) for p, n in zip(prompts, limits)]
    got = [[] for _ in prompts]
    final = {}
    for events in dflash_generate_batch_stream(gen.target.model, gen.draft, prompts, limits, 0.0,
                                               gen.target.stop_token_ids()):
        for ev in events:
            got[ev.index].extend(ev.token_ids)
            if ev.finished:
                final[ev.index] = ev
    for b, s in enumerate(singles):
        assert got[b] == s.generated_tokens, b
        assert final[b].finish_reason == s.metrics["finish_reason"]
        assert final[b].acceptance_lengths == s.metrics["acceptance_lengths"]


def test_openai_batching_runner_concurrent_requests(gen):
    """Three concurrent chat requests decoded as one batch answer like three single requests."""
    import threading

    from dflash_b200.openai_server import BatchingRunner, DFlashRunner
    prompts = ["alpha beta gamma", "one two", "the quick brown fox jumps"]
    single = DFlashRunner(generator=gen)
    want = [single.generate(prompt=p, max_new_tokens=20, temperature=0.0) for p in prompts]
    runner = BatchingRunner(gen, max_batch=8, window_s=0.5)
    got = {}

    def client(i):
        got[i] = runner.generate(prompt=prompts[i], max_new_tokens=20, temperature=0.0)

    threads = [threading.Thread(target=client, args=(i,)) for i in range(3)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    runner.close()
    assert runner.batches == [3]
    for i in range(3):
        assert got[i].text == want[i].text and got[i].completion_tokens == want[i].completion_tokens
        assert got[i].finish_reason == want[i].finish_reason
        assert got[i].prompt_tokens == want[i].prompt_tokens


@pytest.mark.parametrize("n", [0, 1, 2])
def test_short_generations_follow_the_reference_limits(gen, n):
    """max_new_tokens 0, 1, 2 (runtime.py:376-404, 517-521): no generated token at 0 (and no
    token event), else exactly the first n tokens of the plain greedy decode; the stream's
    token events reassemble them and the last event is the finished one."""
    prompt = list(range(9, 30))
    plain = gen.generate_from_tokens(prompt, max_new_tokens=5, speculative_tokens=1)
    res = gen.generate_from_tokens(prompt, max_new_tokens=n)
    assert res.generated_tokens == plain.generated_tokens[:n]
    assert res.metrics["num_output_tokens"] == n
    events = list(gen.stream_from_tokens(prompt, max_new_tokens=n))
    assert [t for e in events for t in e.token_ids] == plain.generated_tokens[:n]
    assert events[-1].finished


def test_one_token_prompt_is_lossless(gen):
    res = gen.generate_from_tokens([17], max_new_tokens=24)
    plain = gen.generate_from_tokens([17], max_new_tokens=24, speculative_tokens=1)
    assert res.output_tokens == plain.output_tokens
    assert len(res.generated_tokens) == 24
