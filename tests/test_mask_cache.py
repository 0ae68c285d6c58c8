"""Allowed-token masks per grammar state (needle_mask_cache_*, include/needle_grammar.h), on the CPU.

The cache must be invisible: for every grammar it is asked about, the mask in its slot holds exactly
the ids a fresh scan returns (needle_grammar_allowed, itself pinned against the reference's
clone-and-feed scan in test_grammar.py).  Walkers that share one template decode side by side with
random choices, so many of them pass through states with equal keys while their texts differ (the
free content of strings, different numbers of array items); every hit is checked against a fresh
scan, which is what catches a key that drops something the grammar still reads (an enum or
uniqueItems around a string, a string constraint, the room left under the 64 KiB limit).
"""
import numpy as np
import pytest

from needle_b200.native import NeedleError

SCHEMAS = [
    # tool-call grammars: (tools, maximum_calls)
    ("tools", None),
    ("tools", [{"name": "lookup", "parameters": {"type": "object", "properties": {
        "query": {"type": "string"}, "limit": {"type": "integer", "minimum": 0, "maximum": 50},
        "mode": {"type": "string", "enum": ["fast", "full"]}, "tags": {"type": "array", "items": {"type": "string"},
                                                                       "uniqueItems": True, "maxItems": 3}},
        "required": ["query"]}},
        {"name": "ping", "parameters": {"type": "object", "properties": {}}}]),
    # JSON-value grammars
    ("schema", {"type": "array", "items": {"type": "string"}, "maxItems": 6}),
    ("schema", {"type": "array", "items": {"type": "string"}, "uniqueItems": True, "maxItems": 4}),
    ("schema", {"type": "array", "items": {"type": "string", "minLength": 2, "maxLength": 5}, "maxItems": 4}),
    ("schema", {"type": "array", "items": {"type": "array", "items": {"type": "string"}},
                "enum": [[["ab"]], [["ab", "c"]], [["x"]]]}),
    ("schema", {"type": "object", "properties": {"k": {"const": "fixed"}, "s": {"type": "string",
                                                                               "pattern": "^[a-z ]*$"},
                                                 "n": {"type": "number"}}, "required": ["k"]}),
    ("schema", {"$defs": {"p": {"type": "object", "properties": {"x": {"type": "integer"},
                                                                  "y": {"$ref": "#/$defs/q"}}},
                          "q": {"type": ["string", "null"]}},
                "type": "array", "items": {"$ref": "#/$defs/p"}, "maxItems": 3}),
]


@pytest.fixture(scope="module")
def G():
    import needle_b200.build
    needle_b200.build.build()
    from needle_b200 import grammar
    return grammar


@pytest.fixture(scope="module")
def vocab(G):
    from needle_b200 import synth
    pieces, types, _ = synth.tokenizer_pieces(8192, 0)
    return G.Vocabulary(pieces, types)


def _template(G, kind, spec):
    if kind == "tools":
        from needle_b200.toolcall import synthetic_tools
        return G.ToolCallGrammar(spec if spec is not None else synthetic_tools(5), 3)
    return G.JsonSchemaGrammar(spec)


def _walk(G, vocab, template, cache, walkers, steps, seed, base_bytes=0, threads=4):
    """Random walkers over one template; every lookup is compared with fresh scans."""
    rng = np.random.default_rng(seed)
    simple = set(b"abcdefghijklmnopqrstuvwxyz0123456789 ")
    gs = [template.clone() for _ in range(walkers)]
    out = [base_bytes + int(rng.integers(0, 24)) if base_bytes else 0 for _ in range(walkers)]
    checked = 0
    for step in range(steps):
        live = [k for k in range(walkers) if gs[k] is not None]
        if not live:
            break
        slots, counts, filled = cache.lookup([gs[k] for k in live], [out[k] for k in live], threads)
        assert len(set(filled.tolist())) == filled.size
        for j, k in enumerate(live):
            fresh = G.allowed(gs[k], vocab, out[k])
            got = cache.ids(int(slots[j]))
            np.testing.assert_array_equal(got, fresh, err_msg=f"walker {k} step {step}")
            assert counts[j] == fresh.size
            checked += 1
            if fresh.size == 0 or gs[k].complete:
                gs[k] = None
                continue
            plain = [i for i in fresh if set(vocab.piece[i]) <= simple]
            short = [i for i in fresh if len(vocab.piece[i]) <= 2]
            r = rng.random()
            pool = plain if plain and r < 0.6 else short if short and r < 0.85 else fresh
            pick = int(pool[rng.integers(0, len(pool))])
            assert gs[k].feed(vocab.piece[pick])
            out[k] += len(vocab.piece[pick])
    return checked


@pytest.mark.parametrize("case", range(len(SCHEMAS)))
def test_cached_masks_equal_fresh_scans(G, vocab, case):
    kind, spec = SCHEMAS[case]
    template = _template(G, kind, spec)
    cache = G.MaskCache(template, vocab, capacity=512)
    checked = _walk(G, vocab, template, cache, walkers=8, steps=40, seed=case)
    stats = cache.stats
    assert checked == stats["hits"] + stats["misses"]
    assert stats["hits"] > 0, stats  # the walkers share their first states at least


def test_free_string_content_shares_one_state(G, vocab):
    """Inside an unconstrained string whose value nothing checks, the text so far is not part of
    the state: walkers with different contents hit one mask."""
    template = G.JsonSchemaGrammar({"type": "array", "items": {"type": "string"}})
    cache = G.MaskCache(template, vocab, capacity=64)
    gs = []
    for text in (b'["abc', b'["hello wor', b'["x", "yy', b'["q'):
        g = template.clone()
        assert g.feed(text.replace(b", ", b","))
        gs.append(g)
    slots, counts, filled = cache.lookup(gs[:2] + gs[3:], [0, 0, 0])
    assert len(set(slots.tolist())) == 1 and filled.size == 1
    # a string whose array checks uniqueness keeps its text in the state
    t2 = G.JsonSchemaGrammar({"type": "array", "items": {"type": "string"}, "uniqueItems": True})
    c2 = G.MaskCache(t2, vocab, capacity=64)
    a, b = t2.clone(), t2.clone()
    assert a.feed(b'["ab') and b.feed(b'["cd')
    s2, _, f2 = c2.lookup([a, b], [0, 0])
    assert s2[0] != s2[1] and f2.size == 2


@pytest.mark.parametrize("schema,texts", [
    # uniqueItems compares the finished strings: `68"]` closes a duplicate in the first
    ({"type": "array", "items": {"type": "string"}, "uniqueItems": True}, [b'["ab68","ab', b'["cd68","ab']),
    # an enum on an enclosing array (an alternative of anyOf, so the value is not a literal choice)
    ({"anyOf": [{"type": "array", "items": {"type": "string"}, "enum": [["ab68"], ["x"]]}, {"type": "integer"}]},
     [b'["ab', b'["cd']),
    # a const on an enclosing object
    ({"anyOf": [{"type": "object", "properties": {"s": {"type": "string"}}, "const": {"s": "ab25"}},
                {"type": "null"}]}, [b'{"s":"ab25', b'{"s":"cd25']),
    # a pattern on the string itself
    ({"type": "array", "items": {"type": "string", "pattern": "^ab"}}, [b'["ab', b'["cd']),
])
def test_checked_contents_stay_in_the_key(G, vocab, schema, texts):
    """Where a later check reads a string's value, states that differ only in the text so far must
    not share a mask (each pair below has different allowed sets)."""
    template = G.JsonSchemaGrammar(schema)
    gs = []
    for t in texts:
        g = template.clone()
        assert g.feed(t), t
        gs.append(g)
    fresh = [G.allowed(g, vocab, 0) for g in gs]
    assert not np.array_equal(fresh[0], fresh[1])  # the case is meaningful
    cache = G.MaskCache(template, vocab, capacity=16)
    slots, counts, _ = cache.lookup(gs, [0, 0])
    assert slots[0] != slots[1]
    for j in range(2):
        np.testing.assert_array_equal(cache.ids(int(slots[j])), fresh[j])


def test_output_limit_is_part_of_the_key(G, vocab):
    template = G.JsonSchemaGrammar({"type": "string"})
    cache = G.MaskCache(template, vocab, capacity=64)
    g = template.clone()
    assert g.feed(b'"ab')
    n_long = len(G.allowed(g, vocab, 0))
    slots, counts, _ = cache.lookup([g, g, g, g], [0, 100, 65_534, 65_536])
    assert slots[0] == slots[1]  # room beyond the longest piece: the same walk
    assert counts[0] == n_long and 0 < counts[2] < n_long and counts[3] == 0
    assert len({int(slots[0]), int(slots[2]), int(slots[3])}) == 3
    np.testing.assert_array_equal(cache.ids(int(slots[2])), G.allowed(g, vocab, 65_534))


def test_near_the_output_limit(G, vocab):
    template = _template(G, "tools", None)
    cache = G.MaskCache(template, vocab, capacity=256)
    assert _walk(G, vocab, template, cache, walkers=6, steps=30, seed=7, base_bytes=65_536 - 60) > 0


def test_eviction_keeps_masks_exact(G, vocab):
    """A table much smaller than the states visited: slots are reused least recently used first and
    every lookup still returns exact masks."""
    template = _template(G, "tools", None)
    cache = G.MaskCache(template, vocab, capacity=8)
    _walk(G, vocab, template, cache, walkers=6, steps=40, seed=11)
    assert cache.stats["evictions"] > 0


def test_capacity_below_one_lookup_and_foreign_grammars(G, vocab):
    template = G.JsonSchemaGrammar({"type": "array", "items": {"type": "integer"}})
    cache = G.MaskCache(template, vocab, capacity=2)
    gs = []
    for text in (b"[", b"[1", b"[12,"):
        g = template.clone()
        assert g.feed(text)
        gs.append(g)
    with pytest.raises(NeedleError) as e:
        cache.lookup(gs, [0, 0, 0])
    assert e.value.code == "INVALID_TOOL_SCHEMA"
    # the failed call left no slot claimed with a mask it did not write
    slots, counts, _ = cache.lookup(gs[:2], [0, 0])
    for j in range(2):
        np.testing.assert_array_equal(cache.ids(int(slots[j])), G.allowed(gs[j], vocab, 0))
    other = G.JsonSchemaGrammar({"type": "array", "items": {"type": "integer"}})  # equal, not a clone
    with pytest.raises(NeedleError):
        cache.lookup([other], [0])
    slots, counts, filled = cache.lookup([None, gs[0]], [0, 0])
    assert slots[0] == -1 and counts[0] == 0 and counts[1] > 0
