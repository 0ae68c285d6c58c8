"""The constrained tool-call grammar (csrc/grammar.cpp through needle_b200.grammar), on the CPU.

The first five tests restate the reference's own grammar tests case for case
(packages/needle.js/tests/grammar.test.ts:7-99: the schema, the accepted and rejected documents,
the clone independence and the tool-call envelope).  The rest pin details the constrained loop
relies on: JSON.stringify-exact enum candidates, numbers, escapes, the 64 KiB output limit, and the
trie walk returning exactly the ids the reference's clone-and-feed scan over the vocabulary accepts
(packages/needle.js/src/tools/agent.ts:165-176).
"""
import json

import numpy as np
import pytest

PARAMETERS = {
    "type": "object",
    "properties": {
        "enabled": {"type": "boolean"},
        "level": {"type": "integer", "minimum": 0, "maximum": 10},
        "mode": {"type": "string", "enum": ["eco", "boost"]},
        "tags": {"type": "array", "items": {"type": "string", "minLength": 1}, "minItems": 1, "maxItems": 3},
        "location": {
            "type": "object",
            "properties": {"lat": {"type": "number"}, "lon": {"type": "number"}},
            "required": ["lat", "lon"],
        },
    },
    "required": ["enabled", "level", "mode", "tags"],
}


@pytest.fixture(scope="module")
def G():
    import needle_b200.build
    needle_b200.build.build()
    from needle_b200 import grammar
    return grammar


def test_accepts_nested_schema_conforming_json(G):
    g = G.JsonSchemaGrammar(PARAMETERS)
    text = '{"mode":"eco","level":3,"enabled":true,"tags":["a","b"],"location":{"lon":2.5,"lat":-1}}'
    for offset in range(0, len(text), 7):  # uneven chunks: resumable strings / numbers / literals
        assert g.feed(text[offset:offset + 7].encode())
    assert g.complete
    assert g.value == {"mode": "eco", "level": 3, "enabled": True, "tags": ["a", "b"],
                       "location": {"lon": 2.5, "lat": -1}}
    assert list(g.value) == ["mode", "level", "enabled", "tags", "location"]  # insertion order


@pytest.mark.parametrize("text", [
    '{"enabled":true,"level":3,"mode":"eco","tags":["x"],"unknown":1}',
    '{"enabled":true,"level":3,"mode":"eco","mode":"boost","tags":["x"]}',
    '{"enabled":true,"level":3,"mode":"eco"}',
    '{"enabled":true,"level":3,"mode":"invalid","tags":["x"]}',
    '{"enabled":true,"level":11,"mode":"eco","tags":["x"]}',
    '{"enabled":true,"level":3,"mode":"eco","tags":[]}',
    '{"enabled":true,"level":3,"mode":"eco","tags":["x"],}',
])
def test_rejects_unknown_duplicate_missing_enum_range(G, text):
    g = G.JsonSchemaGrammar(PARAMETERS)
    assert not (g.feed(text.encode()) and g.complete)


def test_clones_independently(G):
    base = G.JsonSchemaGrammar({"type": "string", "enum": ["alpha", "alpine"]})
    assert base.feed(b'"alp')
    left, right = base.clone(), base.clone()
    assert left.feed(b'ha"') and right.feed(b'ine"')
    assert left.complete and right.complete
    assert left.value == "alpha" and right.value == "alpine"


TOOLS = [
    {"name": "configure", "description": "Configure a device", "parameters": PARAMETERS},
    {"name": "ping", "parameters": {"type": "object", "properties": {}}},
]


def test_accepts_multiple_non_repeated_tool_calls(G):
    g = G.ToolCallGrammar(TOOLS, 2)
    out = ('[{"name":"configure","arguments":{"enabled":false,"level":5,"mode":"boost","tags":["lab"]}},'
           '{"name":"ping","arguments":{}}]')
    assert g.feed(out.encode())
    assert g.complete
    assert g.calls == [
        {"name": "configure", "arguments": {"enabled": False, "level": 5, "mode": "boost", "tags": ["lab"]}},
        {"name": "ping", "arguments": {}},
    ]


@pytest.mark.parametrize("out", ['[{"name":"missing","arguments":{}}]',
                                 '[{"name":"ping","arguments":{}},{"name":"ping","arguments":{}}]'])
def test_rejects_unregistered_and_repeated_tools(G, out):
    g = G.ToolCallGrammar(TOOLS, 3)
    assert not (g.feed(out.encode()) and g.complete)


def test_invalid_tools_raise_invalid_tool_schema(G):
    from needle_b200.native import NeedleError
    for tools in ([], [{"name": "a\"b"}], [{"name": "x"}, {"name": "x"}],
                  [{"name": "t", "parameters": {"type": "object", "properties": {"a": {}}, "required": ["b"]}}],
                  [{"name": "t", "parameters": {"type": "array"}}]):
        with pytest.raises(NeedleError) as e:
            G.ToolCallGrammar(tools)
        assert e.value.code == "INVALID_TOOL_SCHEMA"


def test_values_numbers_escapes(G):
    cases = [
        # a number ends at the byte after it, so a top-level number never completes: wrap them
        ({"type": "array", "items": {"type": "number"}}, b"[-0.5e+3,0]", [-500.0, 0]),
        ({"type": "array", "items": {"type": "integer"}}, b"[42]", [42]),
        ({"type": "string"}, '"a\\u00e9\\n\\"b"'.encode(), "aé\n\"b"),
        ({"type": "string", "maxLength": 2}, '"éé"'.encode(), "éé"),  # code points
        ({"enum": [1.5, None, "x", True]}, b"null", None),
        ({"type": ["null", "boolean"]}, b"false", False),
        ({"type": "array", "items": {"type": "integer"}, "uniqueItems": True}, b"[1,2]", [1, 2]),
    ]
    for schema, text, want in cases:
        g = G.JsonSchemaGrammar(schema)
        assert g.feed(text), (schema, text)
        assert g.complete, (schema, text)
        assert g.value == want, (schema, g.value)
    for schema, text in [({"type": "array", "items": {"type": "integer"}}, b"[1.5]"),
                         ({"type": "array", "items": {"type": "number"}}, b"[01]"),
                         ({"type": "number"}, b"1 "),
                         ({"type": "string", "maxLength": 1}, b'"ab"'), ({"type": "string"}, b'"\xc3\x28"'),
                         ({"type": "array", "items": {"type": "integer"}, "uniqueItems": True}, b"[1,1]"),
                         ({"type": "array", "items": {"type": "number", "multipleOf": 0.5}}, b"[0.3]")]:
        g = G.JsonSchemaGrammar(schema)
        assert not (g.feed(text) and g.complete), (schema, text)


def test_enum_candidates_use_json_stringify(G):
    # JSON.stringify(1e21) == "1e+21", JSON.stringify(0.000001) == "0.000001", 1e-7 -> "1e-7"
    for value, text in [(1e21, b"1e+21"), (1e-6, b"0.000001"), (1e-7, b"1e-7"), (100.0, b"100"), (-2.5, b"-2.5")]:
        g = G.JsonSchemaGrammar({"enum": [value]})
        assert g.feed(text) and g.complete, (value, text)


def _vocab(G):
    from needle_b200 import synth
    pieces, types, _ = synth.tokenizer_pieces(8192, 0)
    return G.Vocabulary(pieces, types)


def test_allowed_equals_clone_and_feed_scan(G):
    """The trie walk returns exactly the ids whose piece a clone of the grammar accepts."""
    v = _vocab(G)
    tools = [{"name": "lookup", "parameters": {"type": "object", "properties": {
                 "query": {"type": "string"}, "limit": {"type": "integer"},
                 "mode": {"type": "string", "enum": ["fast", "full"]}, "strict": {"type": "boolean"}},
                 "required": ["query"]}},
             {"name": "ping", "parameters": {"type": "object", "properties": {}}}]
    g = G.ToolCallGrammar(tools, 2)
    rng = np.random.default_rng(1)
    text = b""
    for step in range(40):
        ids = G.allowed(g, v, len(text))
        scan = [i for i in range(v.size) if v.piece[i] and g.clone().feed(v.piece[i])]
        np.testing.assert_array_equal(ids, np.array(scan, dtype=np.uint32), err_msg=f"step {step}")
        if ids.size == 0 or g.complete:
            break
        pick = int(ids[rng.integers(0, ids.size)])
        assert g.feed(v.piece[pick])
        text += v.piece[pick]
    assert text.startswith(b'[{"name":"')
    batch = G.allowed_batch([g, None, g.clone()], [len(text), 0, len(text)], v, threads=3)
    np.testing.assert_array_equal(batch[0], G.allowed(g, v, len(text)))
    assert batch[1].size == 0
    np.testing.assert_array_equal(batch[2], batch[0])


def test_output_limit(G):
    v = _vocab(G)
    g = G.JsonSchemaGrammar({"type": "string"})
    assert G.allowed(g, v, 65_536).size == 0
    near = G.allowed(g, v, 65_535)
    assert near.size > 0 and all(len(v.piece[i]) == 1 for i in near)


@pytest.mark.parametrize("case", range(5))
def test_walk_shortcuts_equal_clone_and_feed_scan(G, case):
    """String content (the vocabulary-wide index, the closing-quote check, the byte pieces that break
    UTF-8) and number text are walked without feeding every edge: the ids must still be exactly
    those a clone accepts."""
    schema, opening = [
        ({"type": "array", "items": {"type": "string"}, "maxItems": 3}, b'["'),
        ({"type": "object", "properties": {"a": {"type": "string", "maxLength": 6}, "b": {"type": "integer"}}},
         b'{"a":"'),
        ({"type": "object", "properties": {"k": {"type": "string", "minLength": 3, "pattern": "^[a-z0-9 ]*$"},
                                           "n": {"type": "number"}}, "required": ["k"]}, b'{"k":"'),
        ({"type": "array", "items": {"type": "string", "enum": ["ab", "ab cd", "x\u00e9"]}, "uniqueItems": True},
         b'["'),
        ({"type": "array", "items": {"type": "number", "minimum": -5, "maximum": 5000}}, b"[1"),
    ][case]
    v = _vocab(G)
    g = G.JsonSchemaGrammar(schema)
    assert g.feed(opening)
    rng = np.random.default_rng(case)
    text = opening
    simple = set(b"abcdefghijklmnopqrstuvwxyz0123456789 ")
    for step in range(30):
        ids = G.allowed(g, v, len(text))
        scan = [i for i in range(v.size) if v.piece[i] and g.clone().feed(v.piece[i])]
        np.testing.assert_array_equal(ids, np.array(scan, dtype=np.uint32), err_msg=f"{text!r}")
        if ids.size == 0 or g.complete:
            break
        # mostly simple text (so patterns and lengths can still pass), sometimes a piece that closes
        # the current string or number, sometimes anything (bytes that break UTF-8 included)
        closing = [i for i in ids if any(b in v.piece[i] for b in (b'",]' if case == 4 else b'"'))]
        plain = [i for i in ids if set(v.piece[i]) <= simple]
        r = rng.random()
        pool = closing if closing and r < (0.08 if case == 4 else 0.2) else plain if plain and r < 0.8 else ids
        pick = int(pool[rng.integers(0, len(pool))])
        assert g.feed(v.piece[pick])
        text += v.piece[pick]


@pytest.mark.parametrize("case", range(6))
def test_value_starts_equal_clone_and_feed_scan(G, case):
    """At the first byte of a value the walk filters edges by the bytes that can start it (enum
    candidates' first bytes, or its types' first bytes); alternatives, consts, mixed enums, refs and
    nested containers must still give exactly the clone-and-feed ids."""
    schema = [
        {"anyOf": [{"type": "integer"}, {"type": "string", "maxLength": 3}, {"type": "null"}]},
        {"type": "array", "items": {"enum": [1.5, "x", None, True, {"a": 1}, [2]]}, "maxItems": 4},
        {"type": "object", "properties": {"k": {"const": "fixed"}, "n": {"oneOf": [{"type": "boolean"},
                                                                             {"type": "number", "maximum": 9}]}},
         "required": ["k"]},
        {"$defs": {"p": {"type": "object", "properties": {"x": {"type": "integer"}, "y": {"$ref": "#/$defs/q"}}},
                   "q": {"type": ["string", "null"]}},
         "type": "array", "items": {"$ref": "#/$defs/p"}, "maxItems": 3},
        {"type": "array", "items": {"type": "array", "items": {"type": ["integer", "boolean"]}, "maxItems": 3},
         "maxItems": 3},
        {"enum": ["alpha", "beta", 7, False, None]},
    ][case]
    v = _vocab(G)
    g = G.JsonSchemaGrammar(schema)
    rng = np.random.default_rng(100 + case)
    text = b""
    for step in range(30):
        ids = G.allowed(g, v, len(text))
        scan = [i for i in range(v.size) if v.piece[i] and g.clone().feed(v.piece[i])]
        np.testing.assert_array_equal(ids, np.array(scan, dtype=np.uint32), err_msg=f"{text!r}")
        if ids.size == 0 or g.complete:
            break
        short = [i for i in ids if len(v.piece[i]) <= 2]  # small steps visit more value starts
        pool = short if short and rng.random() < 0.7 else ids
        pick = int(pool[rng.integers(0, len(pool))])
        assert g.feed(v.piece[pick])
        text += v.piece[pick]
