"""Float64 restatement of the learner's forward, loss and backward in torch, for the
full-size parity checks on the GPU (the numpy oracle checks the same algebra at sizes it
finishes in seconds; this copy runs the same formulas in float64 on the device so that a
1,048,576-row batch can be checked too). Formulas and conventions are those of
oracle/spo_oracle.py: masking with the most negative finite float32, q == 0 and
pi_old == 0 terms skipped, dz forced to 0 on illegal cells, ReLU mask from the stored
post-ReLU activation.
"""

import torch

NEG_INF = -3.4028234663852886e38


def mlp_forward(params, x):
    acts = []
    h = x
    last = len(params) - 1
    for i, (w, b) in enumerate(params):
        y = h @ w + b
        if i < last:
            y = torch.clamp_min(y, 0.0)
            acts.append(y)
        h = y
    return acts, h


def mlp_backward(params, x, acts, dout, masks=None):
    """Gradients [(dW, db)]; `masks` (optional, one bool tensor per hidden layer) gives
    the ReLU decisions to use instead of acts > 0."""
    grads = [None] * len(params)
    d = dout
    for i in range(len(params) - 1, -1, -1):
        inp = x if i == 0 else acts[i - 1]
        grads[i] = (inp.t() @ d, d.sum(0))
        if i > 0:
            m = masks[i - 1] if masks is not None else acts[i - 1] > 0
            d = (d @ params[i][0].t()) * m
    return grads


def _masked(z, mask):
    return torch.where(mask == 0, torch.full_like(z, NEG_INF), z)


def actor_loss(z, mask, q, z_old, log_alpha, scale):
    zm = _masked(z, mask)
    log_pi = zm - torch.logsumexp(zm, dim=1, keepdim=True)
    pi = torch.softmax(zm, dim=1)
    ce = -torch.where(q != 0, q * torch.where(q != 0, log_pi, 0.0), 0.0).sum(1)
    zo = _masked(z_old, mask)
    lpo = zo - torch.logsumexp(zo, dim=1, keepdim=True)
    po = torch.softmax(zo, dim=1)
    klo = torch.where(po > 0, po * (torch.where(po > 0, lpo, 0.0) - torch.where(po > 0, log_pi, 0.0)),
                      0.0).sum(1)
    alpha = torch.nn.functional.softplus(torch.tensor(float(log_alpha), dtype=torch.float64))
    dz = torch.where(mask == 0, 0.0, ((pi - q) + alpha * (pi - po)) * scale)
    return {"loss": float(scale * (ce + alpha * klo).sum()), "ce": float(scale * ce.sum()),
            "kl_old": float(scale * klo.sum()), "dz": dz}


def value_loss(v, target, scale):
    d = v - target
    return {"loss": float(scale * (0.5 * d * d).sum()), "dv": d * scale}
