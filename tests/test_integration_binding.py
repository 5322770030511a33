"""The Rust binding written out in INTEGRATION.md against include/needle_b200.h.

No Rust toolchain exists in this image, so the binding cannot be compiled
here. This CPU test keeps it honest instead: its `extern "C"` block declares
exactly the functions the header declares (no more, no fewer), each with the
header's number of arguments and a return value exactly when the header's is
not void, and its #[repr(C)] structs list the header's fields in order."""

import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _strip_c_comments(text: str) -> str:
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    return re.sub(r"//[^\n]*", " ", text)


def _header():
    with open(os.path.join(ROOT, "include", "needle_b200.h")) as f:
        text = _strip_c_comments(f.read())
    functions = {}
    for ret, name, args in re.findall(r"([\w\s\*]+?)\s*\b(nb_\w+)\s*\(([^;{]*?)\)\s*;", text):
        args = " ".join(args.split())
        count = 0 if args in ("", "void") else args.count(",") + 1
        functions[name] = (count, ret.split()[-1] != "void" or "*" in ret)
    structs = {}
    for body, name in re.findall(r"typedef\s+struct\s+\w+\s*\{(.*?)\}\s*(\w+)\s*;", text, flags=re.S):
        fields = []
        for statement in body.split(";"):
            words = statement.replace(",", " , ").split()
            if not words:
                continue
            # "uint32_t a, b, c" / "int32_t active_layers[64]" / "float rope_theta"
            names = " ".join(words[1:]).split(",")
            fields += [re.sub(r"\[.*\]", "", n).strip() for n in names if n.strip()]
        structs[name] = fields
    return functions, structs


def _rust_blocks():
    with open(os.path.join(ROOT, "INTEGRATION.md")) as f:
        text = f.read()
    return re.findall(r"```rust\n(.*?)```", text, flags=re.S)


def _rust_extern():
    blocks = [b for b in _rust_blocks() if 'extern "C" {' in b]
    assert len(blocks) == 1, "one Rust block holds the extern \"C\" declarations"
    body = blocks[0].split('extern "C" {', 1)[1].split("\n}", 1)[0]
    functions = {}
    for name, args, rest in re.findall(r"pub fn (nb_\w+)\s*\((.*?)\)\s*(->[^;]*)?;", body, flags=re.S):
        args = " ".join(args.split())
        functions[name] = (0 if not args else args.count(",") + 1, bool(rest))
    structs = {}
    for name, fields in re.findall(r"pub struct (Nb\w+)\s*\{(.*?)\}", blocks[0], flags=re.S):
        structs[name] = re.findall(r"pub (\w+):", fields)
    return functions, structs


def test_extern_block_declares_every_header_function():
    header, _ = _header()
    rust, _ = _rust_extern()
    assert len(header) >= 35
    assert sorted(rust) == sorted(header), (sorted(set(header) - set(rust)), sorted(set(rust) - set(header)))
    for name, (count, returns) in header.items():
        assert rust[name][0] == count, f"{name}: {rust[name][0]} arguments in Rust, {count} in the header"
        assert rust[name][1] == returns, f"{name}: return value differs"


def test_repr_c_structs_match_the_header():
    _, header = _header()
    _, rust = _rust_extern()
    pairs = {"nb_options": "NbOptions", "nb_step_stats": "NbStepStats", "nb_model_config": "NbModelConfig"}
    for c_name, rust_name in pairs.items():
        assert rust[rust_name] == header[c_name], (c_name, rust[rust_name], header[c_name])


def test_engine_seam_is_written_out():
    """The drop-in above the binding: Engine implemented over the device
    session, the generator's loop, and the Model/Session signatures."""
    text = "\n".join(_rust_blocks())
    for needle in ("impl Engine for B200Engine", "fn complete(&mut self, text: &str, max_new_tokens: usize) -> Response",
                   "fn reset(&mut self)", "fn embed(&self, text: &str) -> Option<Vec<f32>>",
                   "pub struct DeviceGenerator", "fn run_turn(", "pub fn with_depth(&self, depth: usize)",
                   "impl Clone for DeviceSession", "ModelError::Depth"):
        assert needle in text, needle


def test_library_exports_every_header_function(native_built):
    import ctypes

    header, _ = _header()
    lib = ctypes.CDLL(native_built)
    missing = [name for name in header if not hasattr(lib, name)]
    assert not missing, missing
