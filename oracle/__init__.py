"""CPU oracle for the recall scorer (test infrastructure only; see
reattention_topk.py). Nothing in the product package imports this."""
