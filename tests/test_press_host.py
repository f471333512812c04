"""Host-side pieces of the press that need no GPU: the decode window, the
decode ratio, the hook dispatch over a quantized cache, the token journal."""

from types import SimpleNamespace
from unittest.mock import Mock

import pytest
import torch

from core_b200 import press as P
from core_b200.journal import CacheMetadata
from core_b200.queries import HiddenStateWindow, decode_positions


def _bisect_ratio(q_len, target):
    """The reference decoding press's ratio search, restated as the check
    (kvpress/kvpress/presses/decoding_press.py:203-245)."""
    if q_len <= target:
        return 0.0
    r = 1.0 - target / q_len
    lo, hi = 0.0, 1.0
    for _ in range(20):
        n = int(q_len * (1 - r))
        if n == target:
            break
        if n > target:
            lo, r = r, (r + hi) / 2
        else:
            hi, r = r, (lo + r) / 2
    return r


@pytest.mark.parametrize("q_len", [5, 17, 100, 333, 4224, 8320, 16512, 131200, 500001])
def test_ratio_keeps_the_same_count_as_the_bisection(q_len):
    for target in sorted({1, 4, q_len // 7, q_len // 2, (3 * q_len) // 4, q_len - 1, q_len}):
        if target < 1:
            continue
        mine = P.ratio_for_kept_count(q_len, target)
        ref = _bisect_ratio(q_len, target)
        assert int(q_len * (1 - mine)) == int(q_len * (1 - ref)) == min(target, q_len) \
            or q_len <= target


def test_window_keeps_the_last_entries_in_order():
    w = HiddenStateWindow(max_entries=4)
    for i in range(10):
        w.append(torch.full((1, 1, 3), float(i)))
        w.trim()
    assert w.n_entries == 4
    assert w.view()[0, :, 0].tolist() == [6.0, 7.0, 8.0, 9.0]


def test_window_counts_entries_not_tokens():
    w = HiddenStateWindow(max_entries=3)
    w.append(torch.arange(6, dtype=torch.float32).view(1, 3, 2))   # a 3-token forward
    for i in range(3):
        w.append(torch.full((1, 1, 2), 100.0 + i))
        w.trim()
    # three entries remain: the 3-token entry has been dropped whole
    assert w.n_entries == 3 and w.n_tokens == 3
    assert w.view()[0, :, 0].tolist() == [100.0, 101.0, 102.0]


def test_window_slides_and_grows_without_losing_tokens():
    w = HiddenStateWindow(max_entries=5)
    seen = []
    for i in range(200):
        n = 1 + (i % 3)
        x = torch.arange(n, dtype=torch.float32).view(1, n, 1) + 1000 * i
        w.append(x)
        seen.append(x[0, :, 0].tolist())
        w.trim()
        want = [v for e in seen[-5:] for v in e]
        assert w.view()[0, :, 0].tolist() == want
        if i % 37 == 36:
            w.clear()
            seen = []


def test_window_of_zero_entries_keeps_nothing():
    w = HiddenStateWindow(max_entries=0)
    w.append(torch.ones(1, 1, 2))
    assert w.n_entries == 1
    w.trim()
    assert w.n_entries == 0 and w.view().shape[1] == 0


def test_decode_positions_end_at_the_current_token():
    kw = {"position_ids": torch.tensor([[700]]), "cache_position": torch.tensor([300])}
    assert decode_positions(kw, 4, "cpu").tolist() == [[697, 698, 699, 700]]
    kw = {"cache_position": torch.tensor([300])}
    assert decode_positions(kw, 2, "cpu").tolist() == [[299, 300]]
    assert decode_positions({}, 2, "cpu") is None


def test_decoding_hook_schedule_with_multi_token_forwards():
    """Compression when the step count reaches the interval, or at once when
    one forward reaches the target size; the window is emptied after each."""
    calls = []

    def compress(module, hs, keys, values, attentions, kwargs):
        calls.append(hs[0, :, 0].tolist())
        return keys[:, :, :2], values[:, :, :2]

    base = SimpleNamespace(compress=compress, compression_ratio=0.0)
    dp = P.DecodingPress(base_press=base, compression_interval=3, target_size=5,
                         hidden_states_buffer_size=8)
    keys = torch.zeros(1, 1, 10, 1)
    cache = SimpleNamespace(layers=[SimpleNamespace(keys=keys, values=keys)])
    mod = SimpleNamespace(layer_idx=0)

    def step(vals, pos):
        hs = torch.tensor(vals, dtype=torch.float32).view(1, -1, 1)
        cache.layers[0].keys = cache.layers[0].values = torch.zeros(1, 1, 10, 1)
        dp.forward_hook(mod, [], {"hidden_states": hs, "past_key_values": cache,
                                  "cache_position": torch.tensor([pos])}, (keys, None))

    step([1.0], 50)
    step([2.0, 3.0], 51)
    assert calls == []
    step([4.0], 53)
    assert calls == [[1.0, 2.0, 3.0, 4.0]] and dp.layer_step_counts[0] == 0
    step([5.0, 6.0, 7.0, 8.0, 9.0], 60)       # q_len >= target_size
    assert calls[-1] == [5.0, 6.0, 7.0, 8.0, 9.0]
    step([1.0], 0)                             # a prefill forward is ignored
    assert len(calls) == 2 and 0 not in dp.hidden_states_buffer


class _ToyQuantLayer:
    """Stand-in for a quantized cache layer: keys kept as integers / 16."""

    axis_key = 0
    axis_value = 0

    def __init__(self, keys, values):
        self._quantized_keys = self._quantize(keys, 0)
        self._quantized_values = self._quantize(values, 0)
        self.keys = torch.zeros(0)
        self.values = torch.zeros(0)
        self.cumulative_length = keys.shape[2]

    def _quantize(self, t, axis):
        return torch.round(t * 16)

    def _dequantize(self, q):
        return q / 16


def test_quantized_cache_write_back(monkeypatch):
    from transformers.cache_utils import QuantizedCache

    class ToyCache(QuantizedCache):
        def __init__(self, layers):
            self.layers = layers

    k = torch.arange(12, dtype=torch.float32).view(1, 1, 12, 1) / 16
    cache = ToyCache([_ToyQuantLayer(k, -k)])
    keys, values = P.read_cache_layer(cache, 0)
    assert torch.equal(keys, k) and torch.equal(values, -k)
    P.write_cache_layer(cache, 0, keys[:, :, 4:], values[:, :, 4:])
    layer = cache.layers[0]
    assert layer.cumulative_length == 8 and layer.keys.numel() == 0
    assert torch.equal(layer._dequantize(layer._quantized_keys), k[:, :, 4:])


def test_journal_grows_and_keeps_unknown_ids():
    md = CacheMetadata()
    md.record(torch.arange(300).view(1, 300) + 1000)          # contiguous prefill
    md.record(torch.tensor([[7]]), torch.tensor([[400]]))      # a gap: 300..399 unknown
    pos, ids, n = md.align(2, 1, 302, torch.device("cpu"))
    assert n == 302 and ids[0, :300].tolist() == list(range(1000, 1300))
    assert ids[0, 300:].tolist() == [-1, -1]
    md.retain(2, torch.tensor([[0, 299, 301]]))
    pos, ids, n = md.align(2, 1, 3, torch.device("cpu"))
    assert pos.tolist() == [[0, 299, 301]] and n == 302
    with pytest.raises(RuntimeError):
        md.align(3, 1, 500, torch.device("cpu"))             # positions never recorded
    with pytest.raises(ValueError):
        md.record(torch.zeros(2, 1, dtype=torch.long))         # batch changed


def test_scorer_reuses_scores_on_non_scoring_layers():
    press = P.COREScorerPress(indexer=torch.nn.Identity(), feature_extractor=SimpleNamespace(),
                              compression_ratio=0.5, scoring_stride=2, scoring_layer_idx=0,
                              n_sink_protect=0)
    raw = torch.arange(8, dtype=torch.float32).view(1, 1, 8).expand(1, 2, 8)
    keys = torch.zeros(1, 2, 8, 2)
    press._ensure_device = Mock()
    press._compute_scores_from_features = Mock(return_value=raw)
    a = press.score(SimpleNamespace(layer_idx=0), torch.zeros(1, 8, 4), keys, keys, None, {})
    b = press.score(SimpleNamespace(layer_idx=1), torch.zeros(1, 8, 4), keys, keys, None, {})
    assert press._compute_scores_from_features.call_count == 1
    assert torch.equal(a, b)
    # a different cache length forgets the memo
    keys2 = torch.zeros(1, 2, 7, 2)
    press._compute_scores_from_features = Mock(return_value=raw[..., :7])
    press.score(SimpleNamespace(layer_idx=1), torch.zeros(1, 7, 4), keys2, keys2, None, {})
    assert press._compute_scores_from_features.call_count == 1
