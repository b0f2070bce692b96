"""Shared builders for tests: synthetic PPO batches and the flattened (non-TPR) oracle."""

from __future__ import annotations

import torch

from bridge_b200.ops.ppo import PPOLossConfig, ppo_loss_reference


def tree_batch(*, n_trees=1, prefix=128, siblings=4, resp=64, vocab=1024, seed=0, device="cpu",
               temperature=1.0, mask_prob=None):
    """Synthetic PPO batch: each tree = shared prompt + `siblings` distinct responses."""
    g = torch.Generator().manual_seed(seed)
    ids, rmask, old, adv, uids = [], [], [], [], []
    for t in range(n_trees):
        p = torch.randint(0, vocab, (prefix,), generator=g)
        for s in range(siblings):
            r = torch.randint(0, vocab, (resp,), generator=g)
            ids.append(torch.cat([p, r]))
            m = torch.ones(resp, dtype=torch.bool)
            if mask_prob is not None:
                m = torch.rand(resp, generator=g) > mask_prob
                m[0] = True
            rmask.append(m)
            adv.append(torch.randn(resp, generator=g))
            old.append(torch.zeros(resp))
            uids.append(f"u{t}")
    batch = {
        "input_ids": ids,
        "response_mask": rmask,
        "old_log_probs": old,
        "advantages": adv,
        "uid": uids,
        "temperature": temperature,
        "dp_size": 1,
    }
    batch["batch_num_tokens"] = int(sum(int(m.sum()) for m in rmask))
    return batch


def nested_tree_batch(*, n_trees=2, prefix=128, branches=2, mid=32, siblings=2, resp=32, vocab=1024, seed=0):
    """Two-level trees: prompt -> ``branches`` shared middle turns -> ``siblings`` responses each.

    The response of a row is its middle turn plus its own tail (all supervised), so internal segments
    below the root own loss terms too."""
    g = torch.Generator().manual_seed(seed)
    ids, rmask, old, adv, uids = [], [], [], [], []
    for t in range(n_trees):
        p = torch.randint(0, vocab, (prefix,), generator=g)
        for b in range(branches):
            m = torch.randint(0, vocab, (mid,), generator=g)
            for s in range(siblings):
                r = torch.randint(0, vocab, (resp,), generator=g)
                ids.append(torch.cat([p, m, r]))
                rmask.append(torch.ones(mid + resp, dtype=torch.bool))
                adv.append(torch.randn(mid + resp, generator=g))
                old.append(torch.zeros(mid + resp))
                uids.append(f"n{t}")
    batch = {"input_ids": ids, "response_mask": rmask, "old_log_probs": old, "advantages": adv, "uid": uids,
             "temperature": 1.0, "dp_size": 1}
    batch["batch_num_tokens"] = int(sum(int(m.sum()) for m in rmask))
    return batch


@torch.no_grad()
def set_old_log_probs(model, batch, *, jitter=0.01, seed=1):
    """old_log_probs = current log-probs minus U(0, jitter) (the config #1 recipe)."""
    lps = flat_log_probs(model, batch)
    g = torch.Generator().manual_seed(seed)
    batch["old_log_probs"] = [lp.float().cpu() - torch.rand(lp.shape, generator=g) * jitter for lp in lps]


def flat_log_probs(model, batch):
    """Per-row response log-probs of the flattened, non-TPR forward (one row at a time)."""
    dev = next(model.parameters()).device
    out = []
    for ids, m in zip(batch["input_ids"], batch["response_mask"]):
        ids = ids.to(dev)
        n = ids.numel()
        pos = torch.arange(n, device=dev)
        h = model(ids, pos, n)
        r = m.numel()
        q = torch.arange(n - r - 1, n - 1, device=dev)
        logits = model.logits(h.index_select(0, q)).float() / float(batch["temperature"])
        lp = torch.log_softmax(logits, -1).gather(1, ids[n - r:, None]).squeeze(1)
        out.append(lp)
    return out


def flat_ppo_loss(model, batch, cfg=PPOLossConfig()):
    lps = flat_log_probs(model, batch)
    x = torch.cat([lp[m.to(lp.device)] for lp, m in zip(lps, batch["response_mask"])])
    old = torch.cat([o[m] for o, m in zip(batch["old_log_probs"], batch["response_mask"])]).to(x.device)
    adv = torch.cat([a[m] for a, m in zip(batch["advantages"], batch["response_mask"])]).to(x.device)
    loss, _ = ppo_loss_reference(x, old, adv, batch["batch_num_tokens"] / batch["dp_size"], cfg)
    return loss, lps


def grads_of(model):
    return {n: (p.main_grad if hasattr(p, "main_grad") else p.grad).detach().float().clone()
            for n, p in model.named_parameters()}


def rel_err(a, b):
    return float((a - b).norm() / (b.norm() + 1e-12))
