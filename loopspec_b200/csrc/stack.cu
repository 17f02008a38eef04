// Instantiations and launch of the persistent stack kernel (stack.cuh), in
// their own translation unit so they compile in parallel with the engine.
#include "stack.cuh"

namespace ls {

namespace {

template <int BN, int HD>
cudaError_t launch_one(const StackLaunch& L, int grid, cudaStream_t stream, bool pdl) {
  constexpr int ST = stk_stages(BN);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kStkThreads);
  cfg.dynamicSmemBytes = StkSmem<BN, ST>::kTotal;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, stack_kernel<BN, ST, HD>, L);
}

template <int BN, int HD>
cudaError_t prepare_one() {
  constexpr int ST = stk_stages(BN);
  return cudaFuncSetAttribute(stack_kernel<BN, ST, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              StkSmem<BN, ST>::kTotal);
}

}  // namespace

cudaError_t stack_prepare() {
  const cudaError_t errs[] = {
      prepare_one<16, 64>(),  prepare_one<16, 128>(),  prepare_one<32, 64>(),  prepare_one<32, 128>(),
      prepare_one<64, 64>(),  prepare_one<64, 128>(),  prepare_one<128, 64>(), prepare_one<128, 128>(),
      prepare_one<256, 64>(), prepare_one<256, 128>()};
  for (cudaError_t e : errs)
    if (e != cudaSuccess) return e;
  return cudaSuccess;
}

size_t stack_smem_bytes(int bn) {
  switch (bn) {
    case 16: return StkSmem<16, stk_stages(16)>::kTotal;
    case 32: return StkSmem<32, stk_stages(32)>::kTotal;
    case 64: return StkSmem<64, stk_stages(64)>::kTotal;
    case 128: return StkSmem<128, stk_stages(128)>::kTotal;
    default: return StkSmem<256, stk_stages(256)>::kTotal;
  }
}

cudaError_t stack_launch(int bn, int hd, const StackLaunch& L, int grid, cudaStream_t stream, bool pdl) {
#define LS_STK(BN)                                                        \
  case BN:                                                                \
    return hd == 64 ? launch_one<BN, 64>(L, grid, stream, pdl) : launch_one<BN, 128>(L, grid, stream, pdl)
  switch (bn) {
    LS_STK(16);
    LS_STK(32);
    LS_STK(64);
    LS_STK(128);
    LS_STK(256);
    default: return cudaErrorInvalidValue;
  }
#undef LS_STK
}

}  // namespace ls
