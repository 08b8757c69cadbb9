"""The speculative decoding loop of the reference's driver (models/qwen35_27b/test/test_dflash.cpp:1046-1530) over
this library's pieces: draft forward -> top-k -> best-first tree -> tree verify -> accept walk -> commit.  Host
orchestration only; every arithmetic step is a C-ABI call (DraftModel, draft_topk, build_ddtree, TreeTarget), none of
which has a fallback."""
import torch

from .ddtree import build_ddtree, draft_topk
from .dflash_draft import DraftDims, DraftModel
from .tree_verify import MAX_NODES, TreeDims, TreeTarget, dequant_q4k

DRAFT_CTX_MAX = 2048          # the draft sees at most this many committed positions (test_dflash.cpp:1083)
CAPTURE_LAYERS_27B = (1, 16, 31, 46, 61)        # qwen35_target_graph.cpp:692-695


class SpecDecoder:
    """target: TreeTarget built with a feature ring whose layer count equals the draft's n_target_layers;
    draft_weights: dict from make_random_draft_weights / a loader, on the GPU.  The draft has no LM head of its own: its
    hidden states go through the target's (`output_w`, Q4_K or bf16)."""

    def __init__(self, target: TreeTarget, target_weights, draft_dims: DraftDims, draft_weights, mask_token_id: int, budget: int = 32,
                 temperature: float = 1.0, chain_seed: bool = True, draft_ctx_max: int = DRAFT_CTX_MAX):
        T: TreeDims = target.dims
        if target.target_feat is None or len(target.capture_layers) != draft_dims.n_target_layers:
            raise ValueError("the target needs a feature ring with one captured layer per draft input layer")
        if draft_dims.hidden != T.hidden:
            raise ValueError("draft and target hidden sizes differ")
        if not 1 <= budget <= MAX_NODES - 1:
            raise ValueError(f"budget must be 1..{MAX_NODES - 1} nodes beside the root")
        self.target, self.tw, self.D = target, target_weights, draft_dims
        self.mask_token_id, self.budget, self.temperature, self.chain_seed = int(mask_token_id), int(budget), float(temperature), bool(chain_seed)
        # A verify writes the rows of ALL its nodes (root + budget) into the ring at (past + t) % cap before the commit keeps
        # the accepted ones.  Once past >= cap those writes land on the oldest positions still in the ring: rows
        # [past - cap, past + budget + 1 - cap).  With at least the root accepted, the next round's window of W positions ends at
        # past + n_acc >= past + 1, so it stays clear of the overwritten rows only while W <= cap - budget.  (The reference
        # has cap 4096 and a window of 2048.)
        self.draft_ctx_max = min(int(draft_ctx_max), target.feat_cap - self.budget)
        if self.draft_ctx_max < 1:
            raise ValueError(f"feature ring of {target.feat_cap} positions is too small for a tree budget of {self.budget}")
        head = target_weights["output_w"]
        self.draft = DraftModel(draft_dims, draft_weights, max_ctx=self.draft_ctx_max, device=target.device, lm_head=head,
                                lm_head_q4k=head.dtype == torch.uint8, vocab=T.vocab)
        self.last_token = None
        self.stats = {"steps": 0, "committed": 0, "tree_nodes": 0}

    # ---- pieces -----------------------------------------------------------------------------------------------
    def embed(self, token_ids: torch.Tensor) -> torch.Tensor:
        """Rows of the target's embedding table as bf16 [n, hidden] (Q4_K rows are dequantised on the GPU)."""
        table = self.tw["token_embd"]
        rows = table.index_select(0, token_ids.to(table.device, torch.long))
        if table.dtype == torch.uint8:
            return dequant_q4k(rows, "bf16").reshape(rows.shape[0], -1).contiguous()
        return rows.contiguous()

    def prefill(self, prompt_ids) -> int:
        """Feed the prompt through the target as chains of at most MAX_NODES tokens (every node accepted), which fills the
        KV cache, the recurrent state and the feature ring; returns the first generated token."""
        ids = torch.as_tensor(prompt_ids, dtype=torch.int32)
        if ids.numel() == 0:
            raise ValueError("empty prompt")
        dev = self.target.device
        nxt = 0
        for s in range(0, ids.numel(), MAX_NODES):
            chunk = ids[s:s + MAX_NODES].to(dev)
            n = int(chunk.numel())
            parents = torch.arange(-1, n - 1, dtype=torch.int32, device=dev)
            am = self.target.verify(chunk, parents)
            path = torch.arange(n, dtype=torch.int32, device=dev)
            result = torch.stack([torch.tensor(n, dtype=torch.int32, device=dev), am[n - 1]]).to(torch.int32)
            self.target.commit(path, result)
            nxt = int(am[n - 1].item())
        self.last_token = nxt
        return nxt

    def step(self):
        """One draft + verify round.  Returns the list of tokens it commits to the output: the accepted drafted tokens
        followed by the target's own next token (which becomes the next round's root)."""
        if self.last_token is None:
            raise RuntimeError("prefill first")
        tgt, D, dev = self.target, self.D, self.target.device
        noise_ids = torch.full((D.q_len,), self.mask_token_id, dtype=torch.int32, device=dev)
        noise_ids[0] = self.last_token
        window = tgt.feature_window(self.draft_ctx_max)
        _, logits = self.draft.forward(self.embed(noise_ids), window if window.shape[0] else None)
        k = 8 if self.budget > D.q_len - 1 else 1                     # test_dflash.cpp:1154
        lp, ids = draft_topk(logits[1:].float(), k, self.temperature)  # row 0 is the known root token
        tree = build_ddtree(lp.cpu().numpy(), ids.cpu().numpy(), self.budget, self.chain_seed)
        tokens = torch.from_numpy(tree.token_ids.copy())
        tokens[0] = self.last_token
        tgt.verify(tokens.to(dev), torch.from_numpy(tree.parents.copy()).to(dev))
        path, result = tgt.accept()
        n_acc = tgt.commit()
        res = result.cpu().tolist()
        accepted = [int(tokens[i]) for i in path[:n_acc].cpu().tolist()]
        self.last_token = int(res[1])
        self.stats["steps"] += 1
        self.stats["committed"] += n_acc
        self.stats["tree_nodes"] += len(tree.parents)
        return accepted[1:] + [self.last_token]

    def generate(self, prompt_ids, max_tokens: int):
        out = [self.prefill(prompt_ids)]
        while len(out) < max_tokens:
            out.extend(self.step())
        return out[:max_tokens]
