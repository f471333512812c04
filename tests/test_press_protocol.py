"""Host-side press behaviour, restating the reference's own protocol tests
(kvpress/tests/test_core_protocol.py:20-74) against core_b200.press, plus the
decode ratio search and the cache-metadata journal."""

from types import SimpleNamespace
from unittest.mock import Mock, patch

import pytest
import torch

from core_b200 import press as P


def test_sink_protection_preserves_memory_allocation():
    for query_length in (8, 1):  # prefill and decode scoring
        press = P.COREScorerPress(indexer=torch.nn.Identity(), feature_extractor=SimpleNamespace(),
                                  compression_ratio=0.5, scoring_layer_idx=-1, n_sink_protect=4)
        raw = torch.zeros(1, 2, 8)
        keys = torch.zeros(1, 2, 8, 2)
        with patch.object(press, "_ensure_device"), patch.object(
                press, "_compute_scores_from_features", return_value=raw):
            selected = press.score(SimpleNamespace(layer_idx=0), torch.zeros(1, query_length, 4),
                                   keys, keys, None, {})
        assert torch.all(selected[:, :, :4] > selected[:, :, 4:])
        torch.testing.assert_close(raw, torch.zeros_like(raw))
        torch.testing.assert_close(press._cached_memory_scores, raw[:, 0])
        mass = press._cached_memory_scores.softmax(-1)[:, 4:].sum()
        assert abs(mass.item() - 0.5) < 1e-6


@pytest.mark.parametrize("interval", [64, 128, 256, 512])
def test_default_buffer_covers_entire_compression_interval(interval):
    press = P.COREDecodingPress(base_press=SimpleNamespace(compress=Mock()),
                                compression_interval=interval, target_size=4096)
    assert press.hidden_states_buffer_size == interval
    keys = torch.zeros(1, 1, 4097, 1)
    cache = SimpleNamespace(layers=[SimpleNamespace(keys=keys, values=keys)])
    with patch.object(press, "compress", return_value=(keys, keys)) as compress, patch(
            "core_b200.press.read_cache_layer", return_value=(keys, keys)):
        for token in range(interval):
            press.forward_hook(SimpleNamespace(layer_idx=0), [], {
                "hidden_states": torch.tensor([[[float(token)]]]),
                "past_key_values": cache,
                "cache_position": torch.tensor([8192 + token]),
            }, (keys, None))
    compress.assert_called_once()
    queries = compress.call_args.args[1]
    torch.testing.assert_close(queries.flatten(), torch.arange(interval).float())


def test_short_explicit_buffer_is_rejected():
    with pytest.raises(ValueError, match="entire compression interval"):
        P.COREDecodingPress(base_press=SimpleNamespace(compress=Mock()), compression_interval=256,
                            target_size=1024, hidden_states_buffer_size=128)


@pytest.mark.parametrize("q_len,target", [(4224, 4096), (8320, 8192), (256, 192), (17, 4), (100, 99)])
def test_target_ratio_search(q_len, target):
    dp = P.DecodingPress(base_press=SimpleNamespace(compress=Mock(), compression_ratio=0.0),
                         compression_interval=128, target_size=target)
    r = dp._find_target_compression_ratio(q_len, target)
    assert int(q_len * (1 - r)) == target
    assert dp._find_target_compression_ratio(10, 10) == 0.0


def test_retained_budget_matches_protocol():
    assert P.retained_budget(16384, 0.75) == 4096
    assert P.retained_budget(5, 0.9) == 4
    with pytest.raises(ValueError):
        P.retained_budget(0, 0.5)


def test_cache_metadata_journal():
    md = P.CacheMetadata()
    md.record(torch.tensor([[5, 6, 7, 8, 9, 10]]))
    pos, ids, n = md.align(0, 1, 6, torch.device("cpu"))
    assert pos.tolist() == [[0, 1, 2, 3, 4, 5]] and ids.tolist() == [[5, 6, 7, 8, 9, 10]] and n == 6
    md.retain(0, torch.tensor([[0, 2, 5]]))
    md.record(torch.tensor([[11, 12]]), torch.tensor([[6, 7]]))
    pos, ids, n = md.align(0, 1, 5, torch.device("cpu"))
    assert pos.tolist() == [[0, 2, 5, 6, 7]] and ids.tolist() == [[5, 7, 10, 11, 12]] and n == 8
    with pytest.raises(RuntimeError):
        md.align(0, 1, 3, torch.device("cpu"))


def test_prefill_decoding_dispatch_and_budget():
    pre = SimpleNamespace(compression_ratio=0.75, compress=Mock(return_value=("pk", "pv")),
                          reset_cache=Mock())
    dec = P.COREDecodingPress(base_press=pre, compression_interval=4, target_size=1)
    dec.compress = Mock(return_value=("dk", "dv"))
    combo = P.COREPrefillDecodingPress(prefilling_press=pre, decoding_press=dec)
    combo.begin_sequence(16384)
    assert dec.target_size == 4096
    hs = torch.zeros(1, 8, 4)
    assert combo.compress(None, hs, 1, 2, None, {"cache_position": torch.tensor([7])}) == ("pk", "pv")
    assert combo.compress(None, hs[:, :1], 1, 2, None, {"cache_position": torch.tensor([9])}) == ("dk", "dv")
    combo.reset_cache()
    pre.reset_cache.assert_called_once()


def test_unsupported_policies_fail_loudly():
    press = P.COREScorerPress(indexer=None, feature_extractor=SimpleNamespace(config=SimpleNamespace()),
                              compression_ratio=0.5, span_block_size=8)
    with pytest.raises(NotImplementedError):
        press._check_policy()


def test_factory_defaults_match_the_standalone_cli():
    """The reference's standalone CLI loads the press with
    decoding_compression_interval=128 and no target or buffer size
    (kvpress/tests/test_core_protocol.py:76-92); the CLI itself is out of
    scope here, but the factory it calls keeps the same defaults, and the
    registry key resolves to it."""
    import inspect
    sig = inspect.signature(P.load_core_prefill_decoding_press)
    assert sig.parameters["decoding_compression_interval"].default == 128
    assert sig.parameters["decoding_target_size"].default is None
    assert sig.parameters["decoding_hidden_states_buffer_size"].default is None
    assert sig.parameters["compression_ratio"].default is None
    assert P.PRESS_REGISTRY["core_full"] is P.load_core_prefill_decoding_press
    # no target size: decode recompression returns to the retained prefill budget
    pre = SimpleNamespace(compression_ratio=0.5, compress=Mock(), reset_cache=Mock())
    dec = P.COREDecodingPress(base_press=pre, compression_interval=128, target_size=1)
    assert dec.hidden_states_buffer_size == 128
    combo = P.COREPrefillDecodingPress(prefilling_press=pre, decoding_press=dec)
    combo.begin_sequence(8192)
    assert dec.target_size == 4096
