"""Multi-GPU data paths on symmetric peer memory: the per-generation heap with its abort word
(``symm``) and the fused data-parallel gradient reduction + optimizer + weight gather
(``dp_fused``)."""
