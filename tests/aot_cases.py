"""Launch signatures the AOT launcher tests emit (shared by the CPU and GPU tests).

Each case: (out_name, kernel_name, signature, constants, options).  The
signature/constants split follows the reference's compile tool usage
(piton/tools/compile.py:3-6): sizes that vary per call are runtime arguments,
tile sizes and unit strides are baked in.
"""

CASES = [
    ("aot_add", "add_kernel", "x_ptr=*fp32,y_ptr=*fp32,output_ptr=*fp32,n_elements=i32", "BLOCK_SIZE=256", {}),
    ("aot_add_qpu", "add_kernel", "x_ptr=*fp32,y_ptr=*fp32,output_ptr=*fp32,n_elements=i32", "BLOCK_SIZE=64",
     {"qpu_rounding": True}),
    ("aot_softmax", "softmax_kernel",
     "output_ptr=*fp32,input_ptr=*fp32,input_row_stride=i32,output_row_stride=i32,n_cols=i32", "BLOCK_SIZE=1024", {}),
    ("aot_matmul", "matmul_kernel",
     "a_ptr=*fp32,b_ptr=*fp32,c_ptr=*fp32,M=i32,N=i32,stride_am=i32,stride_bk=i32,stride_cm=i32",
     "K=512,stride_ak=1,stride_bn=1,stride_cn=1,BLOCK_SIZE_M=8,BLOCK_SIZE_N=64,BLOCK_SIZE_K=4,GROUP_SIZE_M=4", {}),
    ("aot_matmul_rt", "matmul_kernel",
     "a_ptr=*fp32,b_ptr=*fp32,c_ptr=*fp32,M=i32,N=i32,K=i32,stride_am=i32,stride_ak=i32,stride_bk=i32,"
     "stride_bn=i32,stride_cm=i32,stride_cn=i32",
     "BLOCK_SIZE_M=8,BLOCK_SIZE_N=64,BLOCK_SIZE_K=8,GROUP_SIZE_M=8", {}),
    ("aot_matmul_qpu", "matmul_kernel",
     "a_ptr=*fp32,b_ptr=*fp32,c_ptr=*fp32,M=i32,N=i32,stride_am=i32,stride_bk=i32,stride_cm=i32",
     "K=64,stride_ak=1,stride_bn=1,stride_cn=1,BLOCK_SIZE_M=8,BLOCK_SIZE_N=64,BLOCK_SIZE_K=4,GROUP_SIZE_M=4",
     {"qpu_rounding": True}),
    ("aot_dense", "dense_layer_kernel", "x_ptr=*fp32,w_ptr=*fp32,bias_ptr=*fp32,y_ptr=*fp32,M=i32",
     "N=64,K=128,BLOCK_SIZE_M=4,BLOCK_SIZE_N=64,BLOCK_SIZE_K=4,GROUP_SIZE_M=8,ADD_BIAS=1,RELU=1", {}),
    ("aot_attn", "attn_fwd_kernel",
     "Q=*fp32,K=*fp32,V=*fp32,Out=*fp32,sm_scale=fp32,stride_qh=i32,stride_kh=i32,stride_vh=i32,stride_oh=i32",
     "stride_qm=64,stride_kn=64,stride_kk=1,stride_vn=64,stride_om=64,N_CTX=256,HEAD_DIM=64,BLOCK_M=2,"
     "BLOCK_N=16,CAUSAL=1,EVEN_N=1", {}),
    ("aot_softmax_qpu", "softmax_kernel",
     "output_ptr=*fp32,input_ptr=*fp32,input_row_stride=i32,output_row_stride=i32,n_cols=i32", "BLOCK_SIZE=1024",
     {"qpu_rounding": True}),
    ("aot_attn_qpu", "attn_fwd_kernel",
     "Q=*fp32,K=*fp32,V=*fp32,Out=*fp32,sm_scale=fp32,stride_qh=i32,stride_kh=i32,stride_vh=i32,stride_oh=i32",
     "stride_qm=64,stride_kn=64,stride_kk=1,stride_vn=64,stride_om=64,N_CTX=256,HEAD_DIM=64,BLOCK_M=2,"
     "BLOCK_N=16,CAUSAL=1,EVEN_N=1", {"qpu_rounding": True}),
    ("aot_sigmoid", "sigmoid_kernel", "x_ptr=*fp32,out_ptr=*fp32,n=i32", "BLOCK=256", {}),
    ("aot_layernorm", "layernorm_kernel", "x_ptr=*fp32,out_ptr=*fp32,n=i32,eps=fp32", "BLOCK=128", {}),
    ("aot_copy", "copy_kernel", "x_ptr=*fp32,out_ptr=*fp32,n=i32", "BLOCK=256", {}),
    ("aot_mul", "mul_kernel", "x_ptr=*fp32,y_ptr=*fp32,out_ptr=*fp32,n=i32", "BLOCK=256", {}),
    ("aot_fma_qpu", "fma_kernel", "x_ptr=*fp32,y_ptr=*fp32,out_ptr=*fp32,n=i32,alpha=fp32", "BLOCK=64",
     {"qpu_rounding": True}),
    ("aot_scaled_relu", "scaled_relu_kernel", "x_ptr=*fp32,out_ptr=*fp32,n=i32", "alpha=0.5,BLOCK=128", {}),
    ("aot_exp", "sfu_kernel", "x_ptr=*fp32,out_ptr=*fp32,n=i32", "OP=4,BLOCK=512", {}),
    ("aot_log", "log_kernel", "x_ptr=*fp32,out_ptr=*fp32,n=i32", "BLOCK=512", {}),
    ("aot_idiv", "idiv_kernel", "x_ptr=*i32,y_ptr=*i32,q_ptr=*i32,r_ptr=*i32,n=i32", "BLOCK=256", {}),
    ("aot_udiv", "idiv_kernel", "x_ptr=*u32,y_ptr=*u32,q_ptr=*u32,r_ptr=*u32,n=i32", "BLOCK=256", {}),
    ("aot_row_sum", "row_sum_kernel", "x_ptr=*fp32,out_ptr=*fp32,n_cols=i32,stride=i32", "BLOCK_M=8,BLOCK_N=32",
     {}),
    ("aot_row_max", "row_max_kernel", "x_ptr=*fp32,out_ptr=*fp32,n_cols=i32,stride=i32", "BLOCK_M=8,BLOCK_N=32",
     {}),
    ("aot_transpose", "transpose_kernel", "x_ptr=*fp32,out_ptr=*fp32,n_rows=i32,n_cols=i32,stride_x=i32,"
     "stride_out=i32", "BLOCK_M=16,BLOCK_N=16", {}),
    ("aot_life", "life_kernel", "src_ptr=*i32,dst_ptr=*i32,n_rows=i32,n_cols=i32,stride=i32", "BLOCK_R=4,BLOCK_C=16",
     {}),
    ("aot_life_rows", "life_rows_kernel", "src_ptr=*i32,dst_ptr=*i32,n_rows=i32,n_cols=i32,stride=i32",
     "ROWS=32,BLOCK=64", {}),
    ("aot_life_bits", "life_bits_kernel", "src_ptr=*u32,dst_ptr=*u32,n_rows=i32,n_words=i32,stride=i32",
     "ROWS=16,BLOCK=16", {}),
]
