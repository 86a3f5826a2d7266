"""Model definitions: the GPT module, the eager oracle and the sm_100a engine."""
