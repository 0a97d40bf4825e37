"""Prefix hydration store: fingerprints, similarity threshold, reusable token prefix, LRU order (CPU)."""
import hashlib

import pytest

from omnicoder.retrieval.prefix_hydration import PrefixHydrationStore, common_prefix_len, semantic_fingerprint


def test_fingerprint_counts_hashed_words():
    fp = semantic_fingerprint("Sort the list sort", num_buckets=16)
    assert len(fp) == 16 and sum(fp) == 4
    b = int(hashlib.sha1(b"sort").hexdigest(), 16) % 16
    assert fp[b] >= 2  # "Sort" and "sort" land in the same bucket
    assert semantic_fingerprint("", 8) == [0] * 8 and len(semantic_fingerprint("a", 0)) == 1


def test_lookup_threshold_prefix_and_lru():
    st = PrefixHydrationStore(capacity=2, threshold=0.8)
    st.put("write a python function that sorts a list", "kvA", token_ids=[1, 2, 3, 4, 5])
    st.put("explain the rules of chess to a beginner", "kvB", token_ids=[9, 8, 7])
    h = st.lookup("write a python function that sorts a list quickly", token_ids=[1, 2, 3, 6])
    assert h is not None and h.state == "kvA" and h.similarity >= 0.8 and h.reuse_tokens == 3
    assert st.lookup("completely unrelated words here") is None
    # similar text but no shared leading token: nothing to reuse, so no hit
    assert st.lookup("write a python function that sorts a list", token_ids=[4, 2, 3]) is None
    # without token ids the text match alone decides
    assert st.lookup("write a python function that sorts a list").reuse_tokens is None
    # A was used last, so adding C evicts B
    st.put("translate this sentence into french please", "kvC")
    assert len(st) == 2 and st.lookup("explain the rules of chess to a beginner") is None
    assert st.lookup("write a python function that sorts a list").state == "kvA"
    assert common_prefix_len([1, 2], [1, 2, 3]) == 2 and common_prefix_len([], [1]) == 0
    with pytest.raises(ValueError):
        PrefixHydrationStore(capacity=0)
