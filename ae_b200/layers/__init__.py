"""Drop-in mirrors of the reference's ``specmoe.layers`` MoE modules."""
