"""Greedy speculative decoding over two resident models: the verify loop of
examples/spec_decode_70b.rs:213-336 on librq.  A draft model proposes K
tokens one at a time; the target scores [last, d_1 .. d_K] in one forward
(rq_llama_forward_all, M = K+1 rows through the small-M kernels); the
longest prefix the target agrees with is accepted plus the target's own
next token (the bonus); both KV caches are truncated to the accepted
length.  With greedy sampling the output equals the target's greedy
decode, whatever the draft proposes."""
from __future__ import annotations

from collections import deque


class SpecDecoder:
    def __init__(self, target, draft, k: int = 4, adaptive: bool = False, window: int = 4):
        self.target, self.draft = target, draft
        self.k_max = k
        self.adaptive, self.window = adaptive, window
        self.stats = {"target_forwards": 0, "draft_forwards": 0, "accepted": 0, "proposed": 0}

    def generate(self, prompt_ids, max_new_tokens: int) -> list:
        t, d = self.target, self.draft
        prompt = [int(v) for v in prompt_ids]
        _, last = t.forward(prompt, 0, want_logits=False)
        d.forward(prompt, 0, want_logits=False)
        self.stats["target_forwards"] += 1
        self.stats["draft_forwards"] += 1
        out = [last]
        index_pos = len(prompt)
        k_now = self.k_max
        recent: deque = deque()
        while len(out) < max_new_tokens:
            # 1. draft K tokens: inputs last, d_1 .. d_{K-1}
            drafts, cur = [], last
            for j in range(k_now):
                _, tok = d.forward([cur], index_pos + j, want_logits=False)
                drafts.append(tok)
                cur = tok
                self.stats["draft_forwards"] += 1
            # 2. verify [last, d_1 .. d_K] in one target forward
            _, pred = t.forward_all([last] + drafts, index_pos)
            self.stats["target_forwards"] += 1
            # 3. longest accepted prefix, then the bonus token
            accepted = 0
            bonus = pred[k_now]
            for j in range(k_now):
                if pred[j] == drafts[j]:
                    accepted += 1
                else:
                    bonus = pred[j]
                    break
            self.stats["accepted"] += accepted
            self.stats["proposed"] += k_now
            out.extend(drafts[:accepted] + [bonus])
            # 4. caches: every position before the bonus
            if k_now > 0 and accepted == k_now:
                d.forward([drafts[-1]], index_pos + k_now, want_logits=False)
                self.stats["draft_forwards"] += 1
            new_len = index_pos + accepted + 1
            t.truncate_caches(new_len)
            d.truncate_caches(new_len)
            # 5. adaptive K (spec_decode_70b.rs:305-326)
            if self.adaptive:
                recent.append((accepted, k_now))
                if len(recent) > self.window:
                    recent.popleft()
                acc = sum(a for a, _ in recent)
                att = sum(b for _, b in recent)
                rate = acc / att if att else 1.0
                if len(recent) >= 2 and rate < 0.40 and k_now > 0:
                    k_now -= 1
                    recent.clear()
                elif len(recent) >= self.window and rate > 0.70 and k_now < self.k_max:
                    k_now += 1
                    recent.clear()
            index_pos = new_len
            last = bonus
        return out[:max_new_tokens]
