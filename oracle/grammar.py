"""CPU restatement of the reference's grammar crate — TEST INFRASTRUCTURE.

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline use this
module, as the checker of the device token automaton; nothing in the product
imports it. It restates, machine by machine, what the reference's Rust does:

  compile_schema      schema::compile (crates/grammar/src/schema.rs:29-141):
                      JSON schema -> Node ($ref, const, enum, anyOf/oneOf,
                      type lists, string/integer/number/boolean/null/array/object)
  literal_text        serde_json::to_string of a const/enum value (schema.rs:51-53)
  Machine and states  machine.rs: TextState (70-178), NumberState (180-275),
                      LiteralState (277-313), ArrayState (315-400),
                      ObjectState (402-531), Choice (36-50)
  CallGrammar / CallMachine
                      call.rs:33-174, the tool-call wrapper
                      [{"name":"<tool>","arguments":{...}}, ...]
  NameChoice          the Name stage of CallMachine::step alone (call.rs:123-130):
                      the choice is made as soon as an option has ended
  allowed / advance   TokenBytes::allowed / advance (crates/grammar/src/mask.rs:28-49)
  automaton_mask / automaton_advance
                      the same two operations over a byte automaton, the form
                      the device kernels take: transitions[state][byte] = 0
                      rejects the byte; a value with the top bit set rejects it
                      and moves the machine to the state in the low 31 bits;
                      state 0 = no machine
"""
from __future__ import annotations

import copy
import json
import math

import numpy as np

MAX_DEPTH = 12            # schema.rs:5
MAX_ARRAY_ITEMS = 64      # schema.rs:6-7
MAX_NUMBER_CHARS = 20     # machine.rs:5
NAME_PREFIX = b'{"name":"'          # call.rs:8
ARGUMENTS_PREFIX = b',"arguments":'  # call.rs:9
REJECT_MOVES = 0x80000000


# ------------------------------------------------------------------ schema
def literal_text(value) -> str:
    """serde_json::to_string of a JSON value (compact; strings escaped as
    serde_json escapes them; integers as integers; floats in ryu's shortest form)."""
    if value is None:
        return "null"
    if value is True:
        return "true"
    if value is False:
        return "false"
    if isinstance(value, int):
        return str(value)
    if isinstance(value, float):
        return _ryu(value)
    if isinstance(value, str):
        return _quote(value)
    if isinstance(value, list):
        return "[" + ",".join(literal_text(v) for v in value) + "]"
    if isinstance(value, dict):
        return "{" + ",".join(_quote(k) + ":" + literal_text(v) for k, v in value.items()) + "}"
    raise TypeError(type(value))


def _quote(s: str) -> str:
    out = ['"']
    for ch in s:
        c = ord(ch)
        if ch == '"':
            out.append('\\"')
        elif ch == "\\":
            out.append("\\\\")
        elif c < 0x20:
            out.append({8: "\\b", 9: "\\t", 10: "\\n", 12: "\\f", 13: "\\r"}.get(c, "\\u%04x" % c))
        else:
            out.append(ch)
    out.append('"')
    return "".join(out)


def _ryu(x: float) -> str:
    if math.isnan(x) or math.isinf(x):
        return "null"
    r = repr(x)  # the shortest round-trip digits
    mant, _, exp = r.partition("e")
    digits = mant.replace("-", "").replace(".", "")
    neg = x < 0 or (x == 0 and math.copysign(1.0, x) < 0)
    if "." in mant:
        point = mant.replace("-", "").index(".")
    else:
        point = len(mant.replace("-", ""))
    e10 = (int(exp) if exp else 0) + point  # value = 0.digits * 10^e10
    digits = digits.lstrip("0") or "0"
    if digits == "0":
        return "-0.0" if neg else "0.0"
    lead_zeros = len(mant.replace("-", "").replace(".", "")) - len(mant.replace("-", "").replace(".", "").lstrip("0"))
    e10 -= lead_zeros
    digits = digits.rstrip("0") or "0"
    n = len(digits)
    sign = "-" if neg else ""
    if 0 < e10 <= 16:
        if n <= e10:
            return sign + digits + "0" * (e10 - n) + ".0"
        return sign + digits[:e10] + "." + digits[e10:]
    if -5 < e10 <= 0:
        return sign + "0." + "0" * (-e10) + digits
    exponent = e10 - 1
    body = digits[0] + ("." + digits[1:] if n > 1 else "")
    return sign + body + "e" + str(exponent)


class Node:
    def __init__(self, kind, **fields):
        self.kind = kind
        self.__dict__.update(fields)

    def __repr__(self):
        return f"Node({self.kind}, {', '.join(f'{k}={v!r}' for k, v in self.__dict__.items() if k != 'kind')})"

    def __deepcopy__(self, memo):  # schema nodes are immutable: machines share them
        return self


def _get(schema, key):
    return schema.get(key) if isinstance(schema, dict) else None


def _as_u64(v):
    return v if isinstance(v, int) and not isinstance(v, bool) and v >= 0 else None


def _as_f64(v):
    if isinstance(v, bool) or not isinstance(v, (int, float)):
        return None
    return float(v)


def _resolve(schema, root):
    current = schema
    for _ in range(MAX_DEPTH):
        ref = _get(current, "$ref")
        if not isinstance(ref, str) or not ref.startswith("#/"):
            return current
        target = root
        for part in ref[2:].split("/"):
            nxt = _get(target, part)
            if nxt is None:
                return current
            target = nxt
        current = target
    return current


def compile_schema(schema, root=None, depth: int = 0) -> Node:
    root = schema if root is None else root
    schema = _resolve(schema, root)
    if depth > MAX_DEPTH:
        return Node("text", min_chars=0, max_chars=None)
    if isinstance(schema, dict) and "const" in schema:
        return Node("literals", options=[literal_text(schema["const"])])
    enum = _get(schema, "enum")
    if isinstance(enum, list):
        return Node("literals", options=[literal_text(v) for v in enum])
    for key in ("anyOf", "oneOf"):
        variants = _get(schema, key)
        if isinstance(variants, list):
            nodes = [compile_schema(v, root, depth + 1) for v in variants]
            return nodes[0] if len(nodes) == 1 else Node("choice", nodes=nodes)
    kinds = _get(schema, "type")
    if isinstance(kinds, list):
        nodes = []
        for kind in kinds:
            if isinstance(kind, str):
                single = dict(schema)
                single["type"] = kind
                nodes.append(compile_schema(single, root, depth + 1))
        return Node("choice", nodes=nodes)
    kind = kinds if isinstance(kinds, str) else "string"
    if kind == "integer":
        return _integer_node(schema)
    if kind == "number":
        lo = _as_f64(_get(schema, "minimum"))
        lo = lo if lo is not None else _as_f64(_get(schema, "exclusiveMinimum"))
        hi = _as_f64(_get(schema, "maximum"))
        hi = hi if hi is not None else _as_f64(_get(schema, "exclusiveMaximum"))
        return Node("number", min=lo, max=hi)
    if kind == "boolean":
        return Node("boolean")
    if kind == "null":
        return Node("null")
    if kind == "array":
        items = _get(schema, "items")
        node = compile_schema(items, root, depth + 1) if items is not None else Node("text", min_chars=0, max_chars=None)
        mx = _as_u64(_get(schema, "maxItems"))
        return Node("array", items=node, min_items=_as_u64(_get(schema, "minItems")) or 0,
                    max_items=MAX_ARRAY_ITEMS if mx is None else min(mx, MAX_ARRAY_ITEMS))
    if kind == "object":
        required = [r for r in (_get(schema, "required") or []) if isinstance(r, str)] \
            if isinstance(_get(schema, "required"), list) else []
        props = _get(schema, "properties")
        properties = []
        if isinstance(props, dict):
            for name, child in props.items():
                properties.append((name, compile_schema(child, root, depth + 1), name in required))
        return Node("object", properties=properties)
    return Node("text", min_chars=_as_u64(_get(schema, "minLength")) or 0, max_chars=_as_u64(_get(schema, "maxLength")))


def _saturating_i64(x: float) -> int:
    """Rust's `f64 as i64`: truncation toward zero, saturating, NaN -> 0."""
    if math.isnan(x):
        return 0
    if x >= 9.223372036854775807e18:
        return 9223372036854775807
    if x <= -9.223372036854775808e18:
        return -9223372036854775808
    return int(x)


def _integer_node(schema) -> Node:
    """schema.rs:97-104: inclusive bounds rounded inward, exclusive bounds
    moved one past, the tighter of each pair."""
    def f(key):
        return _as_f64(_get(schema, key))

    def rounded(key, fn, shift=0):
        v = f(key)
        return None if v is None else _saturating_i64(fn(v) if math.isfinite(v) else v) + shift

    lower = rounded("minimum", math.ceil)
    upper = rounded("maximum", math.floor)
    lx = rounded("exclusiveMinimum", math.floor, 1)
    ux = rounded("exclusiveMaximum", math.ceil, -1)

    def tighter(a, b, pick):
        if a is not None and b is not None:
            return pick(a, b)
        return a if a is not None else b

    return Node("integer", min=tighter(lower, lx, max), max=tighter(upper, ux, min))


def tool_specs(tools) -> list:
    """call.rs:16-31: (name, arguments node) of every tool with a string name."""
    out = []
    if not isinstance(tools, list):
        return out
    for tool in tools:
        t = _get(tool, "function")
        t = tool if t is None else t
        name = _get(t, "name")
        if not isinstance(name, str):
            continue
        params = t["parameters"] if isinstance(t, dict) and "parameters" in t else {"type": "object", "properties": {}}
        out.append((name, compile_schema(params, params)))
    return out


# ---------------------------------------------------------------- machines
class LiteralState:
    def __init__(self, options: list, alive: list | None = None):
        self.options = [o if isinstance(o, bytes) else o.encode() for o in options]
        self.alive = list(range(len(options))) if alive is None else list(alive)
        self.position = 0

    def __deepcopy__(self, memo):
        other = LiteralState.__new__(LiteralState)
        other.options, other.alive, other.position = self.options, list(self.alive), self.position
        return other

    def step(self, byte: int) -> bool:
        p = self.position
        survivors = [i for i in self.alive if p < len(self.options[i]) and self.options[i][p] == byte]
        if not survivors:
            return False
        self.alive = survivors
        self.position += 1
        return True

    def can_finish(self) -> bool:
        return any(len(self.options[i]) == self.position for i in self.alive)

    def chosen(self):
        for i in self.alive:
            if len(self.options[i]) == self.position:
                return i
        return None


class TextState:
    def __init__(self, min_chars: int, max_chars):
        self.min_chars, self.max_chars = min_chars, max_chars
        self.count, self.opened, self.closed = 0, False, False
        self.escape = None  # None, "slash" or ("u", left)
        self.continuation = 0

    def has_room(self) -> bool:
        return self.max_chars is None or self.count < self.max_chars

    def step(self, b: int) -> bool:
        if self.closed:
            return False
        if not self.opened:
            self.opened = b == 0x22
            return self.opened
        if self.continuation > 0:
            if b & 0xC0 != 0x80:
                return False
            self.continuation -= 1
            return True
        if self.escape == "slash":
            if b in b'"\\/bfnrt':
                self.escape = None
                self.count += 1
                return True
            if b == ord("u"):
                self.escape = ("u", 4)
                return True
            return False
        if isinstance(self.escape, tuple):
            if not (48 <= b <= 57 or 65 <= b <= 70 or 97 <= b <= 102):
                return False
            left = self.escape[1]
            if left == 1:
                self.escape = None
                self.count += 1
            else:
                self.escape = ("u", left - 1)
            return True
        if b == 0x22:
            if self.count < self.min_chars:
                return False
            self.closed = True
            return True
        if b == 0x5C:
            if not self.has_room():
                return False
            self.escape = "slash"
            return True
        if b <= 0x1F:
            return False
        if b <= 0x7F:
            if not self.has_room():
                return False
            self.count += 1
            return True
        for lo, hi, cont in ((0xC2, 0xDF, 1), (0xE0, 0xEF, 2), (0xF0, 0xF4, 3)):
            if lo <= b <= hi:
                if not self.has_room():
                    return False
                self.count += 1
                self.continuation = cont
                return True
        return False

    def can_finish(self) -> bool:
        return self.closed


class NumberState:
    def __init__(self, lo, hi, fractional: bool):
        self.text = b""
        self.min, self.max, self.fractional = lo, hi, fractional

    def step(self, b: int) -> bool:
        if len(self.text) >= MAX_NUMBER_CHARS:
            return False
        self.text += bytes([b])
        if self._viable():
            return True
        self.text = self.text[:-1]
        return False

    def _split(self):
        neg = self.text[:1] == b"-"
        body = self.text[1:] if neg else self.text
        dot = body.find(b".")
        return (neg, body, None) if dot < 0 else (neg, body[:dot], body[dot + 1:])

    def _viable(self) -> bool:
        neg, integer, fraction = self._split()
        for i, b in enumerate(self.text):
            if not (48 <= b <= 57 or (b == 0x2D and i == 0) or (b == 0x2E and self.fractional)):
                return False
        if self.text.count(b".") > 1:
            return False
        if len(integer) > 1 and integer[:1] == b"0":
            return False
        if fraction is not None and (not integer or not all(48 <= b <= 57 for b in fraction)):
            return False
        if neg and self.min is not None and self.min >= 0:
            return False
        if not integer:
            return True
        return self._range(neg, integer, fraction is not None)

    def _range(self, neg: bool, digits: bytes, has_fraction: bool) -> bool:
        try:
            value = float(digits.decode())
        except ValueError:
            value = 0.0
        lower = -math.inf if self.min is None else float(self.min)
        upper = math.inf if self.max is None else float(self.max)
        if has_fraction:
            lo, hi = (-value - 1.0, -value) if neg else (value, value + 1.0)
            return hi >= lower and lo <= upper
        remaining = max(MAX_NUMBER_CHARS - len(self.text), 0)
        for extra in range(min(remaining, 18) + 1):
            scale = 10.0 ** extra
            lo = value * scale
            hi = lo + scale - 1.0
            span_lo, span_hi = (-hi, -lo) if neg else (lo, hi)
            if span_hi >= lower and span_lo <= upper:
                return True
            if self.fractional and extra == 0:
                flo, fhi = (-value - 1.0, -value) if neg else (value, value + 1.0)
                if fhi >= lower and flo <= upper:
                    return True
        return False

    def can_finish(self) -> bool:
        neg, integer, fraction = self._split()
        if not integer or fraction == b"":
            return False
        try:
            value = float(self.text.decode())
        except ValueError:
            value = math.nan
        return (self.min is None or value >= self.min) and (self.max is None or value <= self.max)


class Machine:
    """Machine::new / step / can_finish (machine.rs:7-68)."""

    def __init__(self, node: Node):
        k = node.kind
        self.kind = k
        if k == "text":
            self.state = TextState(node.min_chars, node.max_chars)
        elif k == "integer":
            self.state = NumberState(node.min, node.max, False)
        elif k == "number":
            self.state = NumberState(node.min, node.max, True)
        elif k == "boolean":
            self.state = LiteralState(["true", "false"])
        elif k == "null":
            self.state = LiteralState(["null"])
        elif k == "literals":
            self.state = LiteralState(node.options)
        elif k == "array":
            self.state = ArrayState(node)
        elif k == "object":
            self.state = ObjectState(node)
        elif k == "choice":
            self.state = [Machine(n) for n in node.nodes]
        else:
            raise ValueError(k)

    def step(self, b: int) -> bool:
        if self.kind == "choice":
            survivors = []
            for alt in self.state:
                cand = copy.deepcopy(alt)
                if cand.step(b):
                    survivors.append(cand)
            if not survivors:
                return False
            self.state = survivors
            return True
        return self.state.step(b)

    def can_finish(self) -> bool:
        if self.kind == "choice":
            return any(m.can_finish() for m in self.state)
        return self.state.can_finish()


class ArrayState:
    def __init__(self, node: Node):
        self.items, self.min_items, self.max_items = node.items, node.min_items, node.max_items
        self.count, self.stage, self.item, self.done = 0, "start", None, False

    def __deepcopy__(self, memo):
        other = copy.copy(self)
        other.item = copy.deepcopy(self.item, memo)
        return other

    def _begin(self, b: int) -> bool:
        if self.count >= self.max_items:
            return False
        m = Machine(self.items)
        if not m.step(b):
            return False
        self.count += 1
        self.stage, self.item = "item", m
        return True

    def step(self, b: int) -> bool:
        if self.done:
            return False
        if self.stage == "start":
            if b == ord("["):
                self.stage = "after_open"
                return True
            return False
        if self.stage == "after_open":
            if b == ord("]") and self.min_items == 0:
                self.done = True
                return True
            return self._begin(b)
        if self.stage == "item":
            if self.item.step(b):
                return True
            if not self.item.can_finish():
                return False
            self.stage, self.item = "after_item", None
            return self.step(b)
        if self.stage == "after_item":
            if b == ord(",") and self.count < self.max_items:
                self.stage = "after_comma"
                return True
            if b == ord("]") and self.count >= self.min_items:
                self.done = True
                return True
            return False
        return self._begin(b)  # after_comma

    def can_finish(self) -> bool:
        return self.done


class ObjectState:
    def __init__(self, node: Node):
        self.properties = node.properties
        self.keys = [('"' + name + '"').encode() for name, _, _ in node.properties]
        self.next, self.stage, self.done = 0, ("start",), False

    def __deepcopy__(self, memo):
        other = copy.copy(self)
        other.stage = copy.deepcopy(self.stage, memo)
        return other

    def _candidates(self) -> list:
        out = []
        for i in range(self.next, len(self.properties)):
            out.append(i)
            if self.properties[i][2]:
                break
        return out

    def _can_close(self) -> bool:
        return all(not req for _, _, req in self.properties[self.next:])

    def _begin_key(self, b: int) -> bool:
        cands = self._candidates()
        if not cands:
            return False
        lit = LiteralState(self.keys, cands)
        if not lit.step(b):
            return False
        self.stage = ("key", lit)
        return True

    def step(self, b: int) -> bool:
        if self.done:
            return False
        st = self.stage
        if st[0] == "start":
            if b == ord("{"):
                self.stage = ("before_key", True)
                return True
            return False
        if st[0] == "before_key":
            if b == ord("}") and st[1] and self._can_close():
                self.done = True
                return True
            return self._begin_key(b)
        if st[0] == "key":
            lit = st[1]
            if lit.step(b):
                return True
            prop = lit.chosen()
            if prop is None:
                return False
            self.stage = ("colon", prop)
            return self.step(b)
        if st[0] == "colon":
            if b == ord(":"):
                self.stage = ("value", st[1], None)
                return True
            return False
        if st[0] == "value":
            prop, active = st[1], st[2]
            if active is None:
                fresh = Machine(self.properties[prop][1])
                if fresh.step(b):
                    self.stage = ("value", prop, fresh)
                    return True
                return False
            if active.step(b):
                return True
            if not active.can_finish():
                return False
            self.next = prop + 1
            self.stage = ("after_value",)
            return self.step(b)
        # after_value
        if b == ord(",") and self.next < len(self.properties):
            self.stage = ("before_key", False)
            return True
        if b == ord("}") and self._can_close():
            self.done = True
            return True
        return False

    def can_finish(self) -> bool:
        return self.done


class CallGrammar:
    """CallGrammar (call.rs:33-61): the tools' names (each followed by its
    closing quote) and argument nodes; require_call(permitted)."""

    def __init__(self, tools_json, require_call: bool = False, permitted: list | None = None):
        tools = json.loads(tools_json) if isinstance(tools_json, (str, bytes)) else tools_json
        self.tools = tool_specs(tools)
        self.names = [(name + '"').encode() for name, _ in self.tools]
        self.allow_empty = not require_call
        self.permitted = None if permitted is None else list(permitted)

    def start(self) -> "CallMachine":
        return CallMachine(self)


class CallMachine:
    """CallMachine::step / is_complete (call.rs:77-174)."""

    def __init__(self, grammar: CallGrammar):
        self.grammar = grammar
        self.stage = ("open",)
        self.completed = 0

    def clone(self) -> "CallMachine":
        other = copy.copy(self)
        other.stage = copy.deepcopy(self.stage)
        return other

    def is_complete(self) -> bool:
        return self.stage[0] == "done"

    def _name_literal(self) -> LiteralState:
        g = self.grammar
        allowed = list(range(len(g.tools))) if g.permitted is None else list(g.permitted)
        return LiteralState(g.names, allowed)

    def step(self, b: int) -> bool:
        st = self.stage
        k = st[0]
        if k == "open":
            if b == ord("["):
                self.stage = ("after_open",)
                return True
            return False
        if k == "after_open":
            if b == ord("]") and self.grammar.allow_empty and self.completed == 0:
                self.stage = ("done",)
                return True
            if b == NAME_PREFIX[0]:
                self.stage = ("prefix", 1)
                return True
            return False
        if k == "prefix":
            pos = st[1]
            if pos >= len(NAME_PREFIX) or NAME_PREFIX[pos] != b:
                return False
            pos += 1
            self.stage = ("name", self._name_literal()) if pos == len(NAME_PREFIX) else ("prefix", pos)
            return True
        if k == "name":
            lit = st[1]
            if not lit.step(b):
                return False
            tool = lit.chosen()
            if tool is not None:
                self.stage = ("middle", tool, 0)
            return True
        if k == "middle":
            tool, pos = st[1], st[2]
            if pos >= len(ARGUMENTS_PREFIX) or ARGUMENTS_PREFIX[pos] != b:
                return False
            pos += 1
            self.stage = ("arguments", Machine(self.grammar.tools[tool][1])) if pos == len(ARGUMENTS_PREFIX) \
                else ("middle", tool, pos)
            return True
        if k == "arguments":
            m = st[1]
            if m.step(b):
                if m.can_finish():
                    self.stage = ("close",)
                return True
            return False
        if k == "close":
            if b == ord("}"):
                self.completed += 1
                self.stage = ("after_call",)
                return True
            return False
        if k == "after_call":
            if b == ord(","):
                self.stage = ("prefix", 0)
                return True
            if b == ord("]"):
                self.stage = ("done",)
                return True
            return False
        return False


class NameChoice:
    """The Name stage of CallMachine::step (call.rs:123-130) on its own: the
    literal steps, and as soon as chosen() names an option that has ended the
    call machine leaves the stage — here, the machine is complete and accepts
    nothing more."""

    def __init__(self, options: list, permitted: list | None = None):
        self.literal = LiteralState(options, permitted)
        self.done = False

    def clone(self) -> "NameChoice":
        return copy.deepcopy(self)

    def step(self, b: int) -> bool:
        if self.done or not self.literal.step(b):
            return False
        self.done = self.literal.chosen() is not None
        return True

    def is_complete(self) -> bool:
        return self.done


# ------------------------------------------------------------- token bytes
def _clone(machine):
    return machine.clone() if hasattr(machine, "clone") else copy.deepcopy(machine)


def allowed(pieces: list, machine) -> list:
    """TokenBytes::allowed (mask.rs:28-42)."""
    first_ok: dict = {}
    out = []
    for piece in pieces:
        if not piece:
            out.append(False)
            continue
        first = piece[0]
        if first not in first_ok:
            first_ok[first] = _clone(machine).step(first)
        if not first_ok[first]:
            out.append(False)
            continue
        trial = _clone(machine)
        out.append(all(trial.step(b) for b in piece))
    return out


def advance(pieces: list, machine, token: int) -> bool:
    """TokenBytes::advance (mask.rs:44-49): steps until the first rejected byte."""
    piece = pieces[token] if 0 <= token < len(pieces) else None
    if piece is None:
        return False
    return all(machine.step(b) for b in piece)


def mask_words(flags) -> np.ndarray:
    """Bit t of word t // 32 set where flags[t] (the boundary's mask layout)."""
    bits = np.asarray(flags, dtype=bool)
    pad = (-bits.size) % 32
    bits = np.concatenate([bits, np.zeros(pad, dtype=bool)]).reshape(-1, 32)
    return (bits.astype(np.uint64) << np.arange(32, dtype=np.uint64)).sum(axis=1).astype(np.uint32)


def automaton_mask(transitions: np.ndarray, complete: np.ndarray, pieces: list, state: int, call_end: int) -> list:
    """One sequence's allowed ids over a byte automaton."""
    V = len(pieces)
    if state == 0:
        return [True] * V
    if complete[state]:
        return [t == call_end for t in range(V)]
    out = []
    for piece in pieces:
        if not piece:
            out.append(False)
            continue
        q = state
        for b in piece:
            q = int(transitions[q, b])
            if q == 0 or q & REJECT_MOVES:
                q = 0
                break
        out.append(q != 0)
    return out


def automaton_advance(transitions: np.ndarray, pieces: list, state: int, token: int, start: int, call_start: int,
                      call_end: int) -> int:
    """generator.rs:118-124 over a byte automaton: the piece's bytes step the
    machine until the first rejected one, which leaves the state, or moves it
    where the table's top bit says so."""
    if token == 0xFFFFFFFF:
        return state
    if token == call_start and state == 0:
        return start
    if token == call_end:
        return 0
    if state != 0 and 0 <= token < len(pieces) and pieces[token]:
        for b in pieces[token]:
            q = int(transitions[state, b])
            if q == 0:
                break
            if q & REJECT_MOVES:
                state = q & ~REJECT_MOVES
                break
            state = q
    return state
