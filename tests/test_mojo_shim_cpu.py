"""The Mojo host-layer sources under mojo/networks/ (not compiled: no Mojo toolchain on the
build machine) checked as text against the C ABI: every external_call names an exported
symbol with the argument count the header declares, and every public function of the
reference's networks/ files keeps its name in the shim."""

import os
import re

import pytest

from spo_mojo_b200 import ffi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIM = os.path.join(ROOT, "mojo", "networks")

# the public functions and structs of the reference's networks/ files that the shim keeps
KEEP = {
    "linear.mojo": ["linear_forward", "linear_backward"],
    "mlp.mojo": ["relu", "CriticParams", "zero_critic_params", "CriticCache", "critic_forward",
                 "CriticGrads", "CriticScratch", "critic_backward", "backward_from_dvalue"],
    "actor.mojo": ["zero_actor_params", "actor_logits", "actor_probs", "actor_log_probs", "Actor"],
    "actor_loss.mojo": ["cross_entropy_rows", "entropy_rows", "kl_rows", "actor_backward"],
    "optim.mojo": ["AdamState", "sum_squares", "global_clip_scale", "ema_update", "adam_step"],
}


def _calls(text):
    """(symbol, argument count) of every external_call["spo_...", T](...) in text."""
    out = []
    for m in re.finditer(r'external_call\["(spo_\w+)",\s*[^\]]+\]\(', text):
        depth, i, args, cur = 1, m.end(), [], ""
        while depth:
            c = text[i]
            if c in "([":
                depth += 1
            elif c in ")]":
                depth -= 1
            if depth == 1 and c == ",":
                args.append(cur)
                cur = ""
            elif depth:
                cur += c
            i += 1
        if cur.strip():
            args.append(cur)
        out.append((m.group(1), len(args)))
    return out


def test_shim_calls_match_the_abi():
    declared = set(ffi.header_symbols())
    seen = 0
    for name in sorted(os.listdir(SHIM)):
        if not name.endswith(".mojo"):
            continue
        with open(os.path.join(SHIM, name)) as f:
            for sym, nargs in _calls(f.read()):
                assert sym in declared, (name, sym)
                assert nargs == len(ffi.SIGNATURES[sym][1]), (name, sym, nargs)
                seen += 1
    assert seen >= 15


@pytest.mark.parametrize("fname", sorted(KEEP))
def test_shim_keeps_the_reference_names(fname):
    with open(os.path.join(SHIM, fname)) as f:
        text = f.read()
    for name in KEEP[fname]:
        assert re.search(rf"^(def|struct) {name}\b", text, flags=re.M), (fname, name)
