/* Empty stand-in for an LLVM header. The reference's npl_tensor_ops.cpp
 * includes <llvm/IR/Module.h> (npl_tensor_ops.cpp:3) but uses nothing from it;
 * LLVM is not installed here, so the oracle build points the include at this
 * empty file. Test infrastructure only. */
