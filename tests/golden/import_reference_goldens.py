"""Copy the reference's committed golden tensors for the learner path into tests/golden/ref/.

The reference (josedanielchg/spo-mojo) ships its goldens as raw little-endian float32
files written by numpy ``.tofile()`` plus a ``.txt`` of shapes per family
(``tests/golden_io.mojo:1-25`` reads them). They were produced by the JAX/optax/Stoix
generators under ``tests/golden/gen/`` at ``jax_default_matmul_precision="highest"``.
Those generators cannot run here (no JAX, optax or Stoix), so the files themselves
are the pin: this script copies the families that cover the learner step, unchanged,
and records a SHA-256 manifest so that a later copy can be checked byte for byte.

Families copied (reference generator in brackets):
  linear*   y = xW + b                         [gen_linear.py]
  linbwd*   dW, db, dx                          [gen_linear_backward.py]
  critic_h* critic MLP forward                  [gen_critic.py]
  cbwd_*    critic MLP gradients                [gen_critic_backward.py]
  actor_h*  masked logits and softmax           [gen_actor.py]
  bw_*      actor loss, dz and gradients        [gen_actor_backward.py]
  ce_*      per-row CE, H(q), KL(q||pi)         [gen_ce_loss.py]
  softmax*, logsumexp*, logsoftmax*, wide_*     [gen_softmax.py]
  adam*     clip_by_global_norm + adam (optax)  [gen_adam.py]
  ema*      optax.incremental_update            [gen_ema.py]
  gae*      Stoix truncated GAE                 [gen_gae.py]

Usage (needs the reference checkout; not run by the tests):
    python tests/golden/import_reference_goldens.py <reference checkout>
"""

import hashlib
import os
import shutil
import sys

PREFIXES = ("linear", "linbwd", "critic_h", "cbwd_", "actor_h", "bw_", "ce_",
            "softmax", "logsumexp", "logsoftmax", "wide_", "adam", "ema", "gae")
TXT = ("linear.txt", "linbwd.txt", "critic.txt", "cbwd.txt", "actor.txt",
       "actor_backward.txt", "ce_loss.txt", "softmax.txt", "adam.txt", "ema.txt",
       "gae.txt")


def main(ref_root):
    src = os.path.join(ref_root, "tests", "golden")
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ref")
    os.makedirs(dst, exist_ok=True)
    names = sorted(n for n in os.listdir(src)
                   if (n.endswith(".bin") and n.startswith(PREFIXES)) or n in TXT)
    lines = []
    for n in names:
        shutil.copyfile(os.path.join(src, n), os.path.join(dst, n))
        with open(os.path.join(dst, n), "rb") as f:
            lines.append(f"{hashlib.sha256(f.read()).hexdigest()}  {n}")
    with open(os.path.join(dst, "MANIFEST.sha256"), "w") as f:
        f.write("\n".join(lines) + "\n")
    print(f"copied {len(names)} files into {dst}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: import_reference_goldens.py <root of the reference checkout>")
    main(sys.argv[1])
