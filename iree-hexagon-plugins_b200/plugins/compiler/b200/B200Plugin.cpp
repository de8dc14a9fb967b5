// IREE compiler plugin for the B200 target: the source a maintainer builds
// inside an IREE checkout (it includes IREE's and MLIR's headers and is not
// compiled by this repository's build, which has no IREE). It mirrors the
// reference's plugin shape --
//   * plugins/compiler/hexagon/PluginRegistration.cpp:9-12 (the C entry
//     point IREE's plugin loader calls),
//   * Target/HexagonSession.cpp:32-75 (a DefaultActivated PluginSession that
//     registers a TargetDevice and a TargetBackend under one name),
//   * Target/HexagonTargetDevice.cpp:20-50 (default device target, device
//     match by ID glob),
//   * Target/HexagonTargetBackend.cpp:32-112 (executable target attribute,
//     pass-pipeline hooks, serializeExecutable),
//   * Target/HexagonExecutableSerialization.cpp:622-635 (the executable is
//     embedded as hal.executable.binary with a format and a MIME type)
// -- with the B200 work done by the library every other entry point of this
// repository uses: the backend prints each executable variant's inner module
// (the dispatch functions over interface bindings, after IREE's dispatch
// formation) and hands the text to hxb_compile_mlir
// (include/hxb200_compiler.h), which applies the HMX-equivalent eligibility
// rules, picks the tile plan of every matmul dispatch and serialises the
// dispatch table. Its decision log becomes remarks, its errors become
// diagnostics on the variant and a failed compilation. The same recogniser
// runs on this repository's tests over the dispatch form
// (tests/test_compiler_host.py::test_dispatch_form_of_a_target_backend).
//
// Link against libhxb200.so; no codegen pass pipeline is registered: the
// B200 executable holds references to prebuilt sm_100a kernels, not
// generated code, so the translation pipeline leaves the variant's linalg
// as it is.

#include <memory>
#include <string>

#include "hxb200_compiler.h"
#include "iree/compiler/Dialect/HAL/IR/HALOps.h"
#include "iree/compiler/Dialect/HAL/Target/TargetBackend.h"
#include "iree/compiler/Dialect/HAL/Target/TargetDevice.h"
#include "iree/compiler/Dialect/HAL/Target/TargetRegistry.h"
#include "iree/compiler/PluginAPI/Client.h"
#include "iree/compiler/Utils/OptionUtils.h"
#include "mlir/IR/Builders.h"
#include "mlir/IR/BuiltinAttributes.h"
#include "mlir/IR/BuiltinOps.h"
#include "llvm/Support/raw_ostream.h"

namespace mlir::iree_compiler::b200 {
namespace HAL = mlir::iree_compiler::IREE::HAL;

// Command-line options of the target (--iree-b200-*), the counterpart of
// HexagonOptions (Target/HexagonOptions.h:18-24) plus the dispatch gates.
struct B200Options {
  bool enableMatmul = true;     // like --iree-hexagon-enable-hmx-matmul
  bool enableW8A16 = true;
  bool enableAttention = true;
  int numSMs = 148;             // SM count the tile plans are chosen for

  void bindOptions(OptionsBinder &binder) {
    static llvm::cl::OptionCategory category("B200 (sm_100a) HAL target");
    binder.opt<bool>("iree-b200-enable-matmul", enableMatmul, llvm::cl::cat(category),
                     llvm::cl::desc("Form tcgen05 matmul dispatches for eligible f16 "
                                    "contractions."));
    binder.opt<bool>("iree-b200-enable-w8a16", enableW8A16, llvm::cl::cat(category),
                     llvm::cl::desc("Form int8-weight matmul dispatches."));
    binder.opt<bool>("iree-b200-enable-attention", enableAttention, llvm::cl::cat(category),
                     llvm::cl::desc("Fuse decomposed attention into one dispatch."));
    binder.opt<int>("iree-b200-num-sms", numSMs, llvm::cl::cat(category),
                    llvm::cl::desc("SM count the tile plans are chosen for."));
  }
};

namespace {

constexpr char kBackendName[] = "b200";

class B200TargetBackend final : public HAL::TargetBackend {
 public:
  explicit B200TargetBackend(const B200Options &options) : options(options) {}

  std::string getLegacyDefaultDeviceID() const override { return kBackendName; }

  void getDefaultExecutableTargets(
      MLIRContext *context, StringRef deviceID, DictionaryAttr deviceConfigAttr,
      SmallVectorImpl<HAL::ExecutableTargetAttr> &executableTargetAttrs) const override {
    executableTargetAttrs.push_back(getExecutableTarget(context));
  }

  // #hal.executable.target<"b200", "cuda-sm100a-hxb-v1", {num_sms = ...}>
  HAL::ExecutableTargetAttr getExecutableTarget(MLIRContext *context) const {
    Builder b(context);
    SmallVector<NamedAttribute> config;
    config.push_back(b.getNamedAttr("num_sms", b.getI64IntegerAttr(options.numSMs)));
    config.push_back(b.getNamedAttr("arch", b.getStringAttr("sm_100a")));
    return b.getAttr<HAL::ExecutableTargetAttr>(b.getStringAttr(kBackendName),
                                                b.getStringAttr(HXB_EXECUTABLE_FORMAT),
                                                b.getDictionaryAttr(config));
  }

  void getDependentDialects(DialectRegistry &registry) const override {}

  void buildConfigurationPassPipeline(HAL::ExecutableTargetAttr, OpPassManager &) override {}
  void buildTranslationPassPipeline(HAL::ExecutableTargetAttr, OpPassManager &) override {}
  void buildLinkingPassPipeline(OpPassManager &) override {}

  LogicalResult serializeExecutable(const SerializationOptions &serOptions,
                                    HAL::ExecutableVariantOp variantOp,
                                    OpBuilder &executableBuilder) override {
    ModuleOp inner = variantOp.getInnerModule();
    std::string text;
    {
      llvm::raw_string_ostream os(text);
      OpPrintingFlags flags;
      flags.enableDebugInfo(false).printGenericOpForm(false);
      inner.print(os, flags);
    }
    hxb_compiler_options_t opts;
    hxb_compiler_options_initialize(&opts);
    opts.enable_matmul = options.enableMatmul;
    opts.enable_w8a16 = options.enableW8A16;
    opts.enable_attention = options.enableAttention;
    opts.num_sms = options.numSMs;
    void *blob = nullptr;
    size_t size = 0;
    char *log = nullptr;
    const hxb_status_t status =
        hxb_compile_mlir(text.data(), text.size(), &opts, &blob, &size, &log);
    // every decision of the target, one remark (or error) per line
    StringRef logRef(log ? log : "");
    SmallVector<StringRef> lines;
    logRef.split(lines, '\n', /*MaxSplit=*/-1, /*KeepEmpty=*/false);
    for (StringRef line : lines) {
      if (line.starts_with("error"))
        variantOp.emitError() << line;
      else
        variantOp.emitRemark() << line;
    }
    hxb_compiler_free(log);
    if (status != HXB_OK) {
      hxb_compiler_free(blob);
      return variantOp.emitError()
             << "B200 target: no executable for variant " << variantOp.getSymName();
    }
    // the export ordinals of the variant map to the executable's functions
    // by symbol name (the runtime looks them up the same way)
    auto data = DenseIntElementsAttr::get(
        VectorType::get({static_cast<int64_t>(size)}, executableBuilder.getIntegerType(8)),
        ArrayRef<int8_t>(static_cast<const int8_t *>(blob), size));
    auto binaryOp = HAL::ExecutableBinaryOp::create(executableBuilder, variantOp.getLoc(),
                                                     variantOp.getSymName(),
                                                     variantOp.getTarget().getFormat(), data);
    binaryOp.setMimeTypeAttr(executableBuilder.getStringAttr(HXB_EXECUTABLE_MIME_TYPE));
    hxb_compiler_free(blob);
    return success();
  }

 private:
  const B200Options &options;
};

class B200TargetDevice final : public HAL::TargetDevice {
 public:
  explicit B200TargetDevice(const B200Options &options) : options(options) {}

  HAL::DeviceTargetAttr getDefaultDeviceTarget(
      MLIRContext *context, const HAL::TargetRegistry &targetRegistry) const override {
    Builder b(context);
    SmallVector<HAL::ExecutableTargetAttr> targets;
    if (auto backend = targetRegistry.getTargetBackend(kBackendName))
      backend->getDefaultExecutableTargets(context, kBackendName, b.getDictionaryAttr({}),
                                           targets);
    return HAL::DeviceTargetAttr::get(context, b.getStringAttr(kBackendName), {}, targets);
  }

  // matches runtime devices whose ID starts with "b200" (the driver name of
  // hxb_hal_driver_module_register), as the reference matches "hexagon*"
  Value buildDeviceTargetMatch(Location loc, Value device, HAL::DeviceTargetAttr targetAttr,
                               OpBuilder &builder) const override {
    return HAL::DeviceTargetAttr::buildDeviceIDAndExecutableFormatsMatch(
        loc, device, "b200*", targetAttr.getExecutableTargets(), builder);
  }

 private:
  const B200Options &options;
};

struct B200Session
    : public PluginSession<B200Session, B200Options, PluginActivationPolicy::DefaultActivated> {
  void populateHALTargetDevices(HAL::TargetDeviceList &targets) override {
    targets.add(kBackendName,
                [options = &options]() { return std::make_shared<B200TargetDevice>(*options); });
  }
  void populateHALTargetBackends(HAL::TargetBackendList &targets) override {
    targets.add(kBackendName,
                [options = &options]() { return std::make_shared<B200TargetBackend>(*options); });
  }
};

}  // namespace
}  // namespace mlir::iree_compiler::b200

IREE_DEFINE_COMPILER_OPTION_FLAGS(::mlir::iree_compiler::b200::B200Options);

extern "C" bool iree_register_compiler_plugin_b200(
    mlir::iree_compiler::PluginRegistrar *registrar) {
  registrar->registerPlugin<::mlir::iree_compiler::b200::B200Session>("b200");
  return true;
}
