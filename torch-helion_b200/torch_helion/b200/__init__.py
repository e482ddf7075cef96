"""B200 backend: the C-ABI binding (:mod:`.lib`) and the OpIR runtime (:mod:`.runtime`)."""
