"""Reference baselines on the hot path: the Quest chunk scorer driving Path D
placement (``quest_path_d``) and the KIVI 2-bit cache (``kivi_cache``)."""
