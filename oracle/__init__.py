"""CPU oracle of the verification pass: test infrastructure, never part of the product path.

qwen_oracle restates the reference's numpy fp32 model (tools/reference/qwen_ref.py) for tree-verify
rows; accept restates the reference's acceptance and commit logic. See each module's header for the
file:line it follows and for who may import it.
"""
