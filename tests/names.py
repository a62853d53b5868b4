"""Kernel names shared by the tests (kept free of the oracle so GPU helpers need no oracle import)."""

#: reference shader names the CUDA library implements (the hot path)
HOT_PATH_SHADERS = (
    "add_bias", "bias_relu", "relu", "relu_grad", "relu6", "relu6_grad",
    "leaky_relu", "leaky_relu_grad", "sigmoid", "sigmoid_grad", "add",
    "scale_add", "grad_accum", "bias_grad", "global_avg_pool",
    "global_avg_pool_backward", "softmax", "loss", "softmax_ce_grad",
    "argmax_correct", "accumulate_scalar", "rms", "grad_sq_reduce",
    "grad_norm_final", "sgd", "sgd_clipped", "adam", "batchnorm_mean_var",
    "batchnorm_forward", "batchnorm_backward_reduce", "batchnorm_backward_dx",
    "dice_loss", "dice_loss_sums", "dice_loss_grad",
    "upsample", "upsample_backward", "concat_insert", "slice", "maxpool_forward",
    "maxpool_backward", "conv_reshape", "conv_grad_reshape", "conv_grad_reshape_relu",
)
