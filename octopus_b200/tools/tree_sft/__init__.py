"""Branch-aware supervised fine-tuning on fork trees of logged episodes.

  trees             fork trees from episode logs (tree.json + result.json): the main thread's
                    history at a fork (root), the main thread from the fork to the next fork
                    (join child) and each branch's own turns (branch children)
  encode            chat-template rendering with per-token labels (assistant blocks only)
  build             logs -> encoded JSONL
  train             LoRA SFT, method "tree" (each tree one prefix-tree micro-batch: the root
                    is computed once and shared by every child through the tree attention
                    plan) or method "flat" (one sequence per child, the baseline)
  check_equivalence tree loss == sum of flat losses, value and adapter gradients
  merge_lora        a PEFT adapter folded into an HF checkpoint
  eval_metrics      branch-behaviour metrics of SWE runs

Reference parity (behaviour): `octopus/tools/tree_sft/*.py` (trees, encode, build,
train_tree, train_flat, check_equivalence, merge_lora, eval_metrics).  The reference's tree
forward passes per-layer caches from a root segment into each child; here the shared root
is one prefix-tree micro-batch of the RL trainer (`rl.actor.build_microbatch`), so the same
tree attention kernels, checkpointing and hybrid-layer tree handling serve SFT.
"""
